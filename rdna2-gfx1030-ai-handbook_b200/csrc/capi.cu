// C ABI of librdna2_b200.so: argument validation and dispatch to the kernels.
// Every check here mirrors a Python-side check of the reference
// (rdna2_ops/int8_gemm.py:131-178) so a bad call fails with a status code
// before anything is launched.
#include <cstdint>

#include "../../include/b2_qlinear.h"
#include "b2_common.cuh"
#include "b2_internal.h"

namespace {

constexpr int kAbiVersion = 1;

inline bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }
inline int fail() { return static_cast<int>(cudaErrorInvalidValue); }
inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

bool valid_block(int block, int64_t K) {
  if (block <= 1) return true;
  if (block & (block - 1)) return false;
  if (block > 4096) return false;
  return K % block == 0;
}

int elem_bytes(int kind) { return (kind == b2::kKindBF16 || kind == b2::kKindF16) ? 2 : 1; }

int check_gemm(int kind, const void* a, int64_t lda, const void* b, int64_t ldb, int64_t M, int64_t N,
               int64_t K, const float* a_scale, const float* b_scale, int64_t b_scale_count,
               const void* bias, int bias_dtype, int epilogue, const void* out, int out_dtype,
               int64_t ldc) {
  if (kind < 0 || kind > 3) return fail();
  if (M < 0 || N < 0 || K < 1 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return fail();
  if (kind == b2::kKindI8 && K > 131071) return fail();  // INT32 accumulator bound
  if (M == 0 || N == 0) return 0;
  const int eb = elem_bytes(kind);
  if (!a || !b || !out) return fail();
  if (!aligned16(a) || !aligned16(b)) return fail();
  if (lda < K || ldb < K || (lda * eb) % 16 || (ldb * eb) % 16) return fail();
  if (ldc < N) return fail();
  if (epilogue < 0 || epilogue > 3) return fail();
  if (epilogue == b2::kEpiNone) {
    if (out_dtype != b2::kI32 || kind != b2::kKindI8) return fail();
  } else {
    if (out_dtype < 0 || out_dtype > 2) return fail();
    if (!a_scale || !b_scale) return fail();
    if (b_scale_count != 1 && b_scale_count != N) return fail();
    if (bias && (bias_dtype < 0 || bias_dtype > 2)) return fail();
  }
  return 0;
}

b2::GemmParams make_params(int64_t M, int64_t N, int64_t K, const float* a_scale,
                           const float* b_scale, int64_t b_scale_count, const void* bias,
                           int bias_dtype, int epilogue, void* out, int out_dtype, int64_t ldc) {
  b2::GemmParams p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  const bool raw = epilogue == b2::kEpiNone;
  p.sa = raw ? nullptr : a_scale;
  p.sb = raw ? nullptr : b_scale;
  p.sb_scalar = (!raw && b_scale_count == 1) ? 1 : 0;
  p.bias = raw ? nullptr : bias;
  p.bias_dtype = bias_dtype;
  p.out = out;
  p.out_dtype = out_dtype;
  p.ldc = ldc;
  p.epilogue = epilogue;
  const int ob = (out_dtype == b2::kF16 || out_dtype == b2::kBF16) ? 2 : 4;
  p.vec_ok = aligned16(out) && ((ldc * ob) % 16 == 0);
  return p;
}

}  // namespace

extern "C" {

int b2_version(void) { return kAbiVersion; }

const char* b2_error_string(int status) { return cudaGetErrorString(static_cast<cudaError_t>(status)); }

int b2_sm_count(void) { return b2::device_sm_count(); }

int b2_pair_capacity(void) { return b2::pair_capacity(); }

int b2_set_gemm_path(int path) {
  if (path < 0 || path > 9) return fail();
  b2::set_gemm_path(path);
  return 0;
}

int b2_set_prologue_path(int path) {
  if (path < 0 || path > 2) return fail();
  b2::set_prologue_path(path);
  return 0;
}

int b2_set_w4a16_path(int path) {
  if (path < 0 || path > 2) return fail();
  b2::set_w4a16_path(path);
  return 0;
}

int b2_set_gather_store(int mode) {
  if (mode < 0 || mode > 2) return fail();
  b2::set_gather_store(mode);
  return 0;
}

int b2_act_quant(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int block, int quant,
                 void* q, int64_t ldq, float* scale, void* stream) {
  if (M < 0 || K < 1 || M > INT32_MAX || K > 16384) return fail();
  if (x_dtype < 0 || x_dtype > 5 || x_dtype == 3 || quant < 0 || quant > 2) return fail();
  if (!valid_block(block, K)) return fail();
  if (M == 0) return 0;
  if (!x || !q || !scale || ldx < K || ldq < K) return fail();
  return static_cast<int>(b2::run_act_quant(x, x_dtype, M, K, ldx, block, quant, q, ldq, scale,
                                            static_cast<cudaStream_t>(stream)));
}

int b2_qgemm(int kind, const void* a, int64_t lda, const void* b, int64_t ldb, int64_t M, int64_t N,
             int64_t K, const float* a_scale, const float* b_scale, int64_t b_scale_count,
             const void* bias, int bias_dtype, int epilogue, void* out, int out_dtype, int64_t ldc,
             void* stream) {
  int st = check_gemm(kind, a, lda, b, ldb, M, N, K, a_scale, b_scale, b_scale_count, bias,
                      bias_dtype, epilogue, out, out_dtype, ldc);
  if (st != 0 || M == 0 || N == 0) return st;
  b2::GemmParams p = make_params(M, N, K, a_scale, b_scale, b_scale_count, bias, bias_dtype,
                                 epilogue, out, out_dtype, ldc);
  return static_cast<int>(b2::run_qgemm(kind, a, lda, b, ldb, p, 0, static_cast<cudaStream_t>(stream)));
}

int b2_repack(const void* src, int elem_bytes_, int64_t rows, int64_t cols, int64_t s_row,
              int64_t s_col, void* dst, int64_t ldd, void* stream) {
  if (rows < 0 || cols < 0 || ldd < cols || (elem_bytes_ != 1 && elem_bytes_ != 2)) return fail();
  if (rows == 0 || ldd == 0) return 0;
  if (!src || !dst) return fail();
  return static_cast<int>(b2::run_repack(src, elem_bytes_, rows, cols, s_row, s_col, dst, ldd,
                                         static_cast<cudaStream_t>(stream)));
}

size_t b2_quant_linear_workspace_bytes(int64_t M, int64_t K) {
  if (M <= 0 || K <= 0) return 0;
  return static_cast<size_t>(round_up(M * round_up(K, 16), 256) + round_up(M * 4, 256));
}

}  // extern "C"

int b2::check_gemm_args(int kind, const void* a, int64_t lda, const void* b, int64_t ldb, int64_t M, int64_t N,
                        int64_t K, const float* a_scale, const float* b_scale, int64_t b_scale_count,
                        const void* bias, int bias_dtype, int epilogue, const void* out, int out_dtype,
                        int64_t ldc) {
  return check_gemm(kind, a, lda, b, ldb, M, N, K, a_scale, b_scale, b_scale_count, bias, bias_dtype, epilogue,
                    out, out_dtype, ldc);
}

// Argument check of the fused linear (shared with the gather variant):
// 0 when the call is valid, including every M == 0 or N == 0 call.
int b2::check_quant_linear(int kind, const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int block,
                           const void* w, int64_t ldw, int64_t N, const float* w_scale, int64_t w_scale_count,
                           const void* bias, int bias_dtype, int epilogue, const void* out, int out_dtype,
                           int64_t ldc, const void* workspace, size_t workspace_bytes) {
  if (kind != b2::kKindI8 && kind != b2::kKindE4M3) return fail();
  if (epilogue == b2::kEpiNone) return fail();
  if (M < 0 || K < 1 || K > 16384 || x_dtype < 0 || x_dtype > 2 || !valid_block(block, K)) return fail();
  const int64_t ldq = round_up(K, 16);
  // Validate the GEMM half with the staging buffer standing in for `a`.
  int st = check_gemm(kind, workspace, ldq, w, ldw, M, N, K, w_scale, w_scale, w_scale_count,
                      bias, bias_dtype, epilogue, out, out_dtype, ldc);
  if (st != 0 || M == 0 || N == 0) return st;
  if (!x || ldx < K) return fail();
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0) return fail();
  if (workspace_bytes < b2_quant_linear_workspace_bytes(M, K)) return fail();
  return 0;
}

extern "C" {

int b2_quant_linear(int kind, const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int block,
                    const void* w, int64_t ldw, int64_t N, const float* w_scale,
                    int64_t w_scale_count, const void* bias, int bias_dtype, int epilogue, void* out,
                    int out_dtype, int64_t ldc, void* workspace, size_t workspace_bytes,
                    void* stream) {
  int st = b2::check_quant_linear(kind, x, x_dtype, M, K, ldx, block, w, ldw, N, w_scale, w_scale_count, bias,
                                  bias_dtype, epilogue, out, out_dtype, ldc, workspace, workspace_bytes);
  if (st != 0 || M == 0 || N == 0) return st;
  const int64_t ldq = round_up(K, 16);
  uint8_t* q = static_cast<uint8_t*>(workspace);
  float* sa = reinterpret_cast<float*>(q + round_up(M * ldq, 256));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = b2::run_act_quant(x, x_dtype, M, K, ldx, block, kind == b2::kKindE4M3 ? 1 : 0, q,
                                    ldq, sa, s, /*early_dependents=*/true);
  if (e != cudaSuccess) return static_cast<int>(e);
  b2::GemmParams p = make_params(M, N, K, sa, w_scale, w_scale_count, bias, bias_dtype, epilogue,
                                 out, out_dtype, ldc);
  p.weight_prefetch = 1;  // the prologue just launched writes only q and sa
  return static_cast<int>(b2::run_qgemm(kind, q, ldq, w, ldw, p, 0, s));
}

namespace {
bool w4_shape_ok(int64_t N, int64_t K, int group) {
  if (N <= 0 || K < 64 || K % 64 || N > INT32_MAX || K > INT32_MAX) return false;
  if (group != 32 && group != 64 && group != 128) return false;
  return K % group == 0;
}
}  // namespace

size_t b2_w4a16_tiles_bytes(int64_t N, int64_t K) {
  return w4_shape_ok(N, K, 64) ? b2::w4a16_tiles_bytes(N, K) : 0;
}

size_t b2_w4a16_groups_bytes(int64_t N, int64_t K, int group) {
  return w4_shape_ok(N, K, group) ? b2::w4a16_groups_bytes(N, K, group) : 0;
}

int b2_w4a16_prepare(const void* data, int layout_kn, int order_high, const float* scales, const void* zeros,
                     int64_t N, int64_t K, int group, int dtype, void* tiles, void* groups, void* stream) {
  if (!w4_shape_ok(N, K, group) || (dtype != b2::kF16 && dtype != b2::kBF16)) return fail();
  if (N * K >= (int64_t{1} << 31)) return fail();
  if (!data || !scales || !zeros || !tiles || !groups) return fail();
  return static_cast<int>(b2::run_w4a16_prepare(static_cast<const uint32_t*>(data), layout_kn != 0,
                                                order_high != 0, scales, static_cast<const int32_t*>(zeros), N, K,
                                                group, dtype, static_cast<uint32_t*>(tiles),
                                                static_cast<uint32_t*>(groups), static_cast<cudaStream_t>(stream)));
}

size_t b2_w4a16_workspace_bytes(int64_t M, int64_t N, int64_t K, int group) {
  if (M <= 0 || M > INT32_MAX || !w4_shape_ok(N, K, group)) return 0;
  return b2::w4a16_workspace(M, N, K);
}

int b2_w4a16_gemm(const void* a, int a_dtype, int64_t lda, const void* tiles, const void* groups, int group,
                  int64_t M, int64_t N, int64_t K, const void* bias, int bias_dtype, void* out, int64_t ldo,
                  void* workspace, size_t workspace_bytes, void* stream) {
  if (a_dtype != b2::kF16 && a_dtype != b2::kBF16) return fail();
  if (M < 0 || N < 0 || M > INT32_MAX || M * N >= (int64_t{1} << 31)) return fail();
  if (M == 0 || N == 0) return K >= 64 && K % 64 == 0 ? 0 : fail();
  if (!w4_shape_ok(N, K, group)) return fail();
  if (!a || !tiles || !groups || !out) return fail();
  if (!aligned16(a) || (lda * 2) % 16 || lda < K) return fail();
  if (!aligned16(tiles) || !aligned16(groups) || ldo < N) return fail();
  if (bias && (bias_dtype < 0 || bias_dtype > 2)) return fail();
  const size_t need = b2_w4a16_workspace_bytes(M, N, K, group);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))) return fail();
  return static_cast<int>(b2::run_w4a16(a, a_dtype, lda, tiles, groups, group, M, N, K, bias, bias_dtype, out,
                                        ldo, static_cast<float*>(workspace), workspace_bytes,
                                        static_cast<cudaStream_t>(stream)));
}

size_t b2_w4a8_tiles_bytes(int64_t N, int64_t K) {
  return (N > 0 && K >= 128 && K % 128 == 0 && N <= INT32_MAX && K <= INT32_MAX) ? b2::w4a8_tiles_bytes(N, K) : 0;
}

size_t b2_w4a8_groups_bytes(int64_t N, int64_t K, int group) {
  if (N <= 0 || K < 128 || K % 128 || (group != 32 && group != 64 && group != 128)) return 0;
  return b2::w4a8_groups_bytes(N, K, group);
}

size_t b2_w4a8_workspace_bytes(int64_t M, int64_t K, int group) {
  if (M <= 0 || K < 128 || K % 128 || (group != 32 && group != 64 && group != 128)) return 0;
  return b2::w4a8_workspace(M, K, group);
}

int b2_w4a8_prepare(const void* data, int layout_kn, int order_high, const float* scales, const void* zeros,
                    int64_t N, int64_t K, int group, void* tiles, void* groups, void* stream) {
  if (b2_w4a8_groups_bytes(N, K, group) == 0 || N * K >= (int64_t{1} << 31)) return fail();
  if (!data || !scales || !zeros || !tiles || !groups) return fail();
  if (!aligned16(tiles) || !aligned16(groups)) return fail();
  return static_cast<int>(b2::run_w4a8_prepare(static_cast<const uint32_t*>(data), layout_kn != 0, order_high != 0,
                                               scales, static_cast<const int32_t*>(zeros), N, K, group, tiles,
                                               groups, static_cast<cudaStream_t>(stream)));
}

int b2_w4a8_gemm(const void* a, int64_t lda, const void* tiles, const void* groups, int group, int64_t M,
                 int64_t N, int64_t K, const float* a_scale, const void* bias, int bias_dtype, int integer,
                 void* out, int64_t ldo, void* workspace, size_t workspace_bytes, void* stream) {
  if (M < 0 || N < 0 || M > INT32_MAX || M * N >= (int64_t{1} << 31)) return fail();
  if (b2_w4a8_groups_bytes(N > 0 ? N : 1, K, group) == 0) return fail();
  if (K * 128 * 15 >= (int64_t{1} << 31)) return fail();  // INT32 accumulator bound
  if (M == 0 || N == 0) return 0;
  if (!a || !tiles || !groups || !out || (!integer && !a_scale)) return fail();
  if (!aligned16(a) || lda < K || lda % 16 || !aligned16(tiles) || !aligned16(groups) || ldo < N) return fail();
  if (bias && (bias_dtype < 0 || bias_dtype > 2)) return fail();
  const size_t need = b2_w4a8_workspace_bytes(M, K, group);
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace)) return fail();
  return static_cast<int>(b2::run_w4a8(static_cast<const int8_t*>(a), lda, tiles, groups, group, M, N, K, a_scale,
                                       bias, bias_dtype, integer != 0, out, ldo, workspace,
                                       static_cast<cudaStream_t>(stream)));
}

int b2_fp8_decode(const void* w, int fp8_dtype, int64_t rows, int64_t cols, int64_t ld, int out_dtype,
                  void* out, int64_t ldo, void* stream) {
  if ((fp8_dtype != b2::kE4M3 && fp8_dtype != b2::kE5M2) || (out_dtype != b2::kF32 && out_dtype != b2::kF16))
    return fail();
  if (rows < 0 || cols < 0 || ld < cols || ldo < cols) return fail();
  if (rows == 0 || cols == 0) return 0;
  if (!w || !out) return fail();
  return static_cast<int>(b2::run_fp8_decode(w, fp8_dtype, rows, cols, ld, out_dtype, out, ldo,
                                             static_cast<cudaStream_t>(stream)));
}

int b2_pack_int4(const void* w, int w_dtype, int64_t ldw, int64_t N, int64_t K, int group, int symmetric,
                 int layout_kn, int order_high, void* data, float* scales, void* zeros, void* sums,
                 void* stream) {
  if (w_dtype < 0 || w_dtype > 2 || N < 0 || K < 0 || N > INT32_MAX || K > INT32_MAX) return fail();
  if (group != 32 && group != 64 && group != 128) return fail();
  if (K % group || ldw < K) return fail();
  if (N == 0 || K == 0) return 0;
  if (!w || !data || !scales || !zeros || !sums) return fail();
  return static_cast<int>(b2::run_pack_int4(w, w_dtype, ldw, N, K, group, symmetric != 0, layout_kn != 0,
                                            order_high != 0, static_cast<int32_t*>(data), scales,
                                            static_cast<int32_t*>(zeros), static_cast<int32_t*>(sums),
                                            static_cast<cudaStream_t>(stream)));
}

int b2_unpack_int4(const void* data, int layout_kn, int order_high, const float* scales, const void* zeros,
                   int64_t N, int64_t K, int group, int out_dtype, void* out, void* stream) {
  if (N < 0 || K < 0 || N > INT32_MAX || K > INT32_MAX) return fail();
  if (group != 32 && group != 64 && group != 128) return fail();
  if (K % group) return fail();
  if (out_dtype != b2::kF32 && out_dtype != b2::kF16 && out_dtype != 3) return fail();
  if (N == 0 || K == 0) return 0;
  if (!data || !zeros || !out || (out_dtype != 3 && !scales)) return fail();
  return static_cast<int>(b2::run_unpack_int4(static_cast<const int32_t*>(data), layout_kn != 0,
                                              order_high != 0, scales, static_cast<const int32_t*>(zeros),
                                              N, K, group, out_dtype, out, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
