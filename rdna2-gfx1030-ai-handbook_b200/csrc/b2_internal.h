// Host-side declarations shared by the CUDA translation units of the library.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b2 {

// Most peers one column-parallel gather writes to (8 GPUs per node).
constexpr int kMaxGatherPeers = 7;
// GemmParams::gather: 0 = no gather; peer copies of each staged output unit
// by 16-byte SM stores (kGatherSm) or by TMA stores through per-peer tensor
// maps (kGatherTma).
constexpr int kGatherSm = 1;
constexpr int kGatherTma = 2;
constexpr int kGatherDefault = kGatherTma;

// Arguments of the sharded activation-prologue modes (column-parallel layers
// whose next layer reads whole rows): exchange buffers [world][M] fp32 of
// every rank (amax mode) or this rank's (codes mode), every rank's code
// buffer at this rank's first column (codes mode), and the completion
// signal: slot `rank` of every rank's flag array, this rank's CTA counter.
struct ShardArgs {
  int world = 0;
  int rank = 0;
  float* xchg[kMaxGatherPeers + 1] = {};
  const float* xlocal = nullptr;
  uint8_t* qout[kMaxGatherPeers + 1] = {};
  uint32_t* flag_slot[kMaxGatherPeers + 1] = {};
  uint32_t* done_count = nullptr;
  uint32_t epoch = 0;
  // fused mode (absmax exchange, in-kernel barrier, codes): this rank's own
  // absmax-phase flags to wait on, and the codes phase's signal
  const uint32_t* own_flags = nullptr;
  uint32_t* flag_slot2[kMaxGatherPeers + 1] = {};
  uint32_t* done_count2 = nullptr;
  uint32_t epoch2 = 0;
  int* status = nullptr;  // the bounded-wait status word
};

struct GemmParams {
  int M, N, K;
  int tiles_m, tiles_n, num_kb;
  const float* sa;     // [M] per-row scale; nullptr for raw accumulators
  const float* sb;     // [N] per-channel scale, or [1] when sb_scalar
  int sb_scalar;
  const void* bias;    // [N] or nullptr
  int bias_dtype;
  void* out;
  int out_dtype;
  int64_t ldc;         // output row stride in elements
  int epilogue;
  int vec_ok;          // output rows 16-byte aligned: vector stores allowed
  int* status;         // device status word for bounded waits
  // Split-K kernel only: stream the first ring of weights before
  // griddepcontrol.wait.  Set only by the fused linear, whose preceding
  // kernel (its own activation prologue) never writes the weights; any other
  // caller's previous kernel may, and its writes are visible only after the wait.
  int weight_prefetch;
  // Column-parallel output gather (b2_quant_linear_gather; pair TMA-store
  // kernel only).  Besides its TMA store of `out`, the epilogue writes every
  // staged 32-row x 128-byte output unit to the n_peers buffers peer_out[i]
  // (other GPUs' full outputs, mapped into this process and offset to this
  // rank's columns; row stride ldc) with plain 16-byte stores over NVLink.
  // The last CTA to finish (counted in *done_count, which it leaves at zero)
  // then stores `epoch` with release semantics at system scope into each of
  // flag_slot[0..n_peers] -- this rank's slot in every rank's flag array, its
  // own included -- after a system-scope fence in every epilogue thread.
  int gather;
  int n_peers;
  void* peer_out[kMaxGatherPeers];
  uint32_t* flag_slot[kMaxGatherPeers + 1];
  uint32_t* done_count;
  uint32_t epoch;
};

// Argument check of the GEMM on quantized operands (b2_qgemm): 0 when
// valid, including every M == 0 or N == 0 call.
int check_gemm_args(int kind, const void* a, int64_t lda, const void* b, int64_t ldb, int64_t M, int64_t N,
                    int64_t K, const float* a_scale, const float* b_scale, int64_t b_scale_count,
                    const void* bias, int bias_dtype, int epilogue, const void* out, int out_dtype, int64_t ldc);

// Argument check of the fused linear (b2_quant_linear): 0 when valid,
// including every M == 0 or N == 0 call; the gather variant shares it.
int check_quant_linear(int kind, const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int block,
                       const void* w, int64_t ldw, int64_t N, const float* w_scale, int64_t w_scale_count,
                       const void* bias, int bias_dtype, int epilogue, const void* out, int out_dtype,
                       int64_t ldc, const void* workspace, size_t workspace_bytes);

// Device address of the bounded-wait status word on the current device.
int* status_word_ptr();

int device_sm_count();

// a: [M,K] K-major with row stride lda (elements); b: [N,K] K-major, ldb.
// Both base pointers 16-byte aligned, lda/ldb * element size multiples of 16.
cudaError_t run_qgemm(int kind, const void* a, int64_t lda, const void* b, int64_t ldb,
                      GemmParams p, int max_ctas, cudaStream_t stream);

// 0 = automatic, 1 = single-CTA kernel only, 2 = 2-CTA pair kernel only.
void set_gemm_path(int path);
void set_gather_store(int mode);
void set_prologue_path(int path);
void set_w4a16_path(int path);
int pair_capacity();

// Per-row rotate + quantize (quant 0 = int8 /127 RNE, 1 = e4m3 /448, 2 = the
// reference row quantizer: int8, half away from zero, step floor 1e-20).
// early_dependents: let the next kernel in the stream (the fused linear's
// GEMM, launched with programmatic serialization) start its setup and
// weight loads while this one runs; only for callers whose next kernel reads
// nothing else this kernel's predecessors may still write.
// One sharded prologue launch (mode 1 = amax exchange, 2 = codes, 3 = both
// with an in-kernel cross-GPU barrier between them, cooperative launch)
// over a column slice [M, Ns] of 16/32-bit activations; Ns may be 0 for
// modes 1 and 2.
cudaError_t run_shard_quant(int mode, const void* y, int y_dtype, int64_t M, int64_t Ns, int64_t ldy, int block,
                            int quant, int64_t ldq, float* scale, const ShardArgs& sh, cudaStream_t stream);

cudaError_t run_act_quant(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx,
                          int block, int quant, void* q, int64_t ldq, float* scale,
                          cudaStream_t stream, bool early_dependents = false);

cudaError_t run_fp8_decode(const void* w, int fp8_dtype, int64_t rows, int64_t cols, int64_t ld,
                           int out_dtype, void* out, int64_t ldo, cudaStream_t stream);

// dst[r, c] = src[r*s_row + c*s_col] for c < cols, 0 for cols <= c < ldd.
cudaError_t run_repack(const void* src, int elem_bytes, int64_t rows, int64_t cols, int64_t s_row,
                       int64_t s_col, void* dst, int64_t ldd, cudaStream_t stream);

// W4A16 on the tiled weight format (see w4a16.cu); `partial` holds the
// stream-K slots, w4a16_workspace(M, N, K) bytes (0 when not needed).
cudaError_t run_w4a16(const void* a, int a_dtype, int64_t lda, const void* tiles, const void* groups, int group,
                      int64_t M, int64_t N, int64_t K, const void* bias, int bias_dtype, void* out, int64_t ldo,
                      float* partial, size_t partial_bytes, cudaStream_t stream);
size_t w4a16_workspace(int64_t M, int64_t N, int64_t K);
size_t w4a16_tiles_bytes(int64_t N, int64_t K);
size_t w4a16_groups_bytes(int64_t N, int64_t K, int group);
cudaError_t run_w4a16_prepare(const uint32_t* data, int layout_kn, int order_high, const float* scales,
                              const int32_t* zeros, int64_t N, int64_t K, int group, int dtype, uint32_t* tiles,
                              uint32_t* groups, cudaStream_t stream);
// W4A8 grouped linear on the W4A8 tile format (see w4a8.cu); workspace holds
// the per-group activation sums, w4a8_workspace(M, K, group) bytes.
size_t w4a8_tiles_bytes(int64_t N, int64_t K);
size_t w4a8_groups_bytes(int64_t N, int64_t K, int group);
size_t w4a8_workspace(int64_t M, int64_t K, int group);
cudaError_t run_w4a8_prepare(const uint32_t* data, int layout_kn, int order_high, const float* scales,
                             const int32_t* zeros, int64_t N, int64_t K, int group, void* tiles, void* groups,
                             cudaStream_t stream);
cudaError_t run_w4a8(const int8_t* a, int64_t lda, const void* tiles, const void* groups, int group, int64_t M,
                     int64_t N, int64_t K, const float* a_scale, const void* bias, int bias_dtype, int integer,
                     void* out, int64_t ldo, void* workspace, cudaStream_t stream);
cudaError_t run_pack_int4(const void* w, int w_dtype, int64_t ldw_el, int64_t N, int64_t K, int G,
                          int symmetric, int layout_kn, int order_high, int32_t* data, float* scales,
                          int32_t* zeros, int32_t* sums, cudaStream_t stream);
cudaError_t run_unpack_int4(const int32_t* data, int layout_kn, int order_high, const float* scales,
                            const int32_t* zeros, int64_t N, int64_t K, int G, int out_dtype, void* out,
                            cudaStream_t stream);

}  // namespace b2
