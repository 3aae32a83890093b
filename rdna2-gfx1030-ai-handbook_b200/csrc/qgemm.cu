// Quantized GEMM with fused dequant epilogue for sm_100a.
//
// C[m,n] = epilogue( sum_k A[m,k] * B[n,k] )  with A [M,K] and B [N,K] both
// K-major (B is the weight in its stored [N,K] layout, i.e. the reference's
// `weight.T` view of rdna2_ops/int8_gemm.py:39-40 without a copy).
//
// Design (one persistent CTA per SM, 192 threads):
//   warp 0      TMA producer: 128B-swizzled A/B k-blocks into a STAGES-deep
//               shared-memory ring (plain tile loads, never multicast).
//   warp 1      TMEM owner + single-thread tcgen05.mma issuer (kind::i8 for
//               W8A8, kind::f8f6f4 for e4m3, kind::f16 for bf16), 128 x BN
//               tiles, 4 MMAs (32 bytes of K each) per k-block.
//   warps 2..5  epilogue: tcgen05.ld of the 128 x BN accumulator (double
//               buffered in TMEM so tile t+1's MMAs overlap tile t's
//               epilogue), per-token x per-channel scale, bias and cast, then
//               direct 16-byte global stores.
//
// Epilogue rounding follows the reference exactly:
//   separate  float(acc)*(sa*sb) then + bias in fp32, two roundings
//             (rdna2_ops/int8_gemm.py:53-63 with enable_fp_fusion=False)
//   fma       fma(float(acc), sa*sb, bias)       (rounding="fused", :191)
//   kitchen   (float(acc)*(sa*sb)).to(out) + bias.to(out)
//             (production/MOSS_RDNA2_INT8/backend.py:128-143)
//   none      raw INT32 accumulator              (int8_matmul, :195-200)
#include <mutex>

#define B2_STATUS_OWNER 1
#include "b2_common.cuh"
#include "b2_internal.h"

namespace b2 {

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int kABytes = 128 * 128;
  static constexpr int kBBytes = BN * 128;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kOffA = 0;
  static constexpr int kOffB = STAGES * kABytes;
  static constexpr int kOffBar = STAGES * kStageBytes;
  static constexpr int kNumBars = 2 * STAGES + 4;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kBytes = kOffMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
  static constexpr uint32_t kTmemCols = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64
                                        : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
};

template <int OUT>
__device__ __forceinline__ float round_through(float v) {
  if constexpr (OUT == kF16) return __half2float(__float2half_rn(v));
  if constexpr (OUT == kBF16) return __bfloat162float(__float2bfloat16_rn(v));
  return v;
}

template <int KIND>
__device__ __forceinline__ float acc_to_float(uint32_t r) {
  if constexpr (KIND == kKindI8) return __int2float_rn(static_cast<int>(r));
  return __uint_as_float(r);
}

template <int KIND, int MODE, int OUT>
__device__ __forceinline__ float epi_value(uint32_t r, float sa, float sb, float bias, bool has_bias) {
  const float acc = acc_to_float<KIND>(r);
  const float s = __fmul_rn(sa, sb);
  if constexpr (MODE == kEpiSeparate) {
    float v = __fmul_rn(acc, s);
    return has_bias ? __fadd_rn(v, bias) : v;
  } else if constexpr (MODE == kEpiFma) {
    return has_bias ? __fmaf_rn(acc, s, bias) : __fmul_rn(acc, s);
  } else {
    float v = round_through<OUT>(__fmul_rn(acc, s));
    return has_bias ? round_through<OUT>(__fadd_rn(v, bias)) : v;
  }
}

__device__ __forceinline__ uint32_t pack2(float a, float b, int out) {
  if (out == kF16) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// One thread, one output row, 32 consecutive columns starting at n.
template <int KIND, int MODE, int OUT>
__device__ __forceinline__ void store_chunk(const GemmParams& p, const uint32_t (&r)[32], int row,
                                            int n, float sa, float sb_lane, float bias_lane,
                                            bool has_bias) {
  // All 32 lanes run the shuffles; rows past M only skip the stores.
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float sbj = p.sb_scalar ? sb_lane : __shfl_sync(0xffffffffu, sb_lane, j);
    const float bj = __shfl_sync(0xffffffffu, bias_lane, j);
    if constexpr (MODE == kEpiNone) {
      v[j] = __uint_as_float(r[j]);
    } else {
      v[j] = epi_value<KIND, MODE, OUT>(r[j], sa, sbj, bj, has_bias);
    }
  }
  if (row >= p.M) return;
  const int64_t base = static_cast<int64_t>(row) * p.ldc + n;
  if (p.vec_ok && n + 32 <= p.N) {
    if constexpr (OUT == kF32 || OUT == kI32) {
      uint4* dst = reinterpret_cast<uint4*>(static_cast<uint32_t*>(p.out) + base);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        dst[j] = make_uint4(__float_as_uint(v[4 * j]), __float_as_uint(v[4 * j + 1]),
                            __float_as_uint(v[4 * j + 2]), __float_as_uint(v[4 * j + 3]));
    } else {
      uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + base);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        dst[j] = make_uint4(pack2(v[8 * j], v[8 * j + 1], OUT), pack2(v[8 * j + 2], v[8 * j + 3], OUT),
                            pack2(v[8 * j + 4], v[8 * j + 5], OUT),
                            pack2(v[8 * j + 6], v[8 * j + 7], OUT));
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (n + j < p.N) {
        if constexpr (OUT == kF32 || OUT == kI32) {
          static_cast<uint32_t*>(p.out)[base + j] = __float_as_uint(v[j]);
        } else if constexpr (OUT == kF16) {
          static_cast<__half*>(p.out)[base + j] = __float2half_rn(v[j]);
        } else {
          static_cast<__nv_bfloat16*>(p.out)[base + j] = __float2bfloat16_rn(v[j]);
        }
      }
    }
  }
}

template <int KIND>
__device__ __forceinline__ void store_dispatch(const GemmParams& p, const uint32_t (&r)[32], int row,
                                               int n, float sa, float sb_lane, float bias_lane) {
  const bool hb = p.bias != nullptr;
  switch (p.epilogue * 4 + p.out_dtype) {
    case kEpiNone * 4 + kI32: store_chunk<KIND, kEpiNone, kI32>(p, r, row, n, sa, sb_lane, bias_lane, hb); break;
    case kEpiSeparate * 4 + kF32: store_chunk<KIND, kEpiSeparate, kF32>(p, r, row, n, sa, sb_lane, bias_lane, hb); break;
    case kEpiSeparate * 4 + kF16: store_chunk<KIND, kEpiSeparate, kF16>(p, r, row, n, sa, sb_lane, bias_lane, hb); break;
    case kEpiSeparate * 4 + kBF16: store_chunk<KIND, kEpiSeparate, kBF16>(p, r, row, n, sa, sb_lane, bias_lane, hb); break;
    case kEpiFma * 4 + kF32: store_chunk<KIND, kEpiFma, kF32>(p, r, row, n, sa, sb_lane, bias_lane, hb); break;
    case kEpiFma * 4 + kF16: store_chunk<KIND, kEpiFma, kF16>(p, r, row, n, sa, sb_lane, bias_lane, hb); break;
    case kEpiFma * 4 + kBF16: store_chunk<KIND, kEpiFma, kBF16>(p, r, row, n, sa, sb_lane, bias_lane, hb); break;
    case kEpiKitchen * 4 + kF32: store_chunk<KIND, kEpiKitchen, kF32>(p, r, row, n, sa, sb_lane, bias_lane, hb); break;
    case kEpiKitchen * 4 + kF16: store_chunk<KIND, kEpiKitchen, kF16>(p, r, row, n, sa, sb_lane, bias_lane, hb); break;
    case kEpiKitchen * 4 + kBF16: store_chunk<KIND, kEpiKitchen, kBF16>(p, r, row, n, sa, sb_lane, bias_lane, hb); break;
    default: break;
  }
}

template <int KIND, int BN, int STAGES>
__global__ void __launch_bounds__(192, 1)
    qgemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                 const GemmParams p) {
  using L = GemmSmem<BN, STAGES>;
  constexpr int kKbElems = (KIND == kKindBF16) ? 64 : 128;  // 128 bytes of K per k-block
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);

  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = p.tiles_m * p.tiles_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int tm = tile % p.tiles_m, tn = tile / p.tiles_m;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kSiteProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
          tma_load_2d(&tma_a, &full[stage], smem + L::kOffA + stage * L::kABytes, kb * kKbElems,
                      tm * 128);
          tma_load_2d(&tma_b, &full[stage], smem + L::kOffB + stage * L::kBBytes, kb * kKbElems,
                      tn * BN);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc<KIND>(128, BN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int t = 0;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++t) {
        const int buf = t & 1;
        const uint32_t use = static_cast<uint32_t>(t >> 1);
        if (!mbar_wait(&tempty[buf], (use & 1u) ^ 1u, abort_flag, kSiteMmaTmem)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * BN);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, kSiteMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + L::kOffA + stage * L::kABytes);
          const uint32_t b_addr = smem_u32(smem + L::kOffB + stage * L::kBBytes);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma<KIND>(d_tmem, sw128_desc(a_addr + kk * 32), sw128_desc(b_addr + kk * 32), idesc,
                       (kb | kk) != 0 ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[buf]);
      }
    }
  } else {
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    int t = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++t) {
      const int buf = t & 1;
      const uint32_t use = static_cast<uint32_t>(t >> 1);
      const int tm = tile % p.tiles_m, tn = tile / p.tiles_m;
      const int row = tm * 128 + quarter * 32 + lane;
      const float sa = (p.sa != nullptr && row < p.M) ? p.sa[row] : 0.0f;
      bool ok = mbar_wait(&tfull[buf], use & 1u, abort_flag, kSiteEpilogue);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(buf * BN);
      const float sb_scalar = (p.sb != nullptr && p.sb_scalar) ? p.sb[0] : 0.0f;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        const int n = tn * BN + c * 32;
        // Lane j carries column n+j's scale and bias; store_chunk broadcasts.
        float sb_lane = sb_scalar, bias_lane = 0.0f;
        if (n + lane < p.N) {
          if (p.sb != nullptr && !p.sb_scalar) sb_lane = p.sb[n + lane];
          if (p.bias != nullptr) {
            bias_lane = load_as_float(p.bias, p.bias_dtype, n + lane);
            if (p.epilogue == kEpiKitchen) {
              if (p.out_dtype == kF16) bias_lane = round_through<kF16>(bias_lane);
              if (p.out_dtype == kBF16) bias_lane = round_through<kBF16>(bias_lane);
            }
          }
        }
        uint32_t r[32];
        tmem_ld32(taddr + static_cast<uint32_t>(c * 32), r);
        tmem_ld_wait(r);
        if (c == BN / 32 - 1) {
          // Accumulator fully read: hand the TMEM buffer back to the MMA warp.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[buf]);
        }
        store_dispatch<KIND>(p, r, row, n, sa, sb_lane, bias_lane);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// ----------------------------------------------------------------- host side

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encoder() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 2-D K-major operand map: dims {inner (K elements), rows}, 128-byte swizzle,
// box {128 bytes of K, box_rows}; out-of-range elements read as zero.
static cudaError_t make_kmajor_map(CUtensorMap* map, const void* ptr, int elem_bytes, int64_t inner,
                                   int64_t rows, int64_t row_stride_bytes, int box_rows) {
  EncodeTiledFn fn = encoder();
  if (fn == nullptr) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride_bytes)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / elem_bytes),
                             static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, elem_bytes == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16,
                  2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  static int cache[64] = {0};
  if (dev < 64 && cache[dev] > 0) return cache[dev];
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (n <= 0) n = 148;
  if (dev < 64) cache[dev] = n;
  return n;
}

template <int KIND, int BN, int STAGES>
static cudaError_t launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, GemmParams p,
                               int max_ctas, cudaStream_t stream) {
  using L = GemmSmem<BN, STAGES>;
  auto kernel = qgemm_kernel<KIND, BN, STAGES>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  p.tiles_n = static_cast<int>((p.N + BN - 1) / BN);
  const int tiles = p.tiles_m * p.tiles_n;
  int grid = device_sm_count();
  if (max_ctas > 0 && max_ctas < grid) grid = max_ctas;
  if (tiles < grid) grid = tiles;
  if (grid <= 0) return cudaSuccess;
  kernel<<<grid, 192, L::kAlloc, stream>>>(ma, mb, p);
  return cudaGetLastError();
}

// Pick the N tile so a persistent wave stays full: wide tiles (more operand
// reuse per MMA) unless they leave most SMs idle.
static int choose_bn(int64_t M, int64_t N) {
  const int64_t tm = (M + 127) / 128;
  const int sms = device_sm_count();
  if (N <= 128) return 128;
  if (tm * ((N + 255) / 256) >= sms) return 256;
  return tm * ((N + 127) / 128) > tm * ((N + 255) / 256) ? 128 : 256;
}

cudaError_t run_qgemm(int kind, const void* a, int64_t lda, const void* b, int64_t ldb, GemmParams p,
                      int max_ctas, cudaStream_t stream) {
  if (p.M == 0 || p.N == 0) return cudaSuccess;
  const int eb = kind == kKindBF16 ? 2 : 1;
  const int bn = choose_bn(p.M, p.N);
  CUtensorMap ma, mb;
  cudaError_t e = make_kmajor_map(&ma, a, eb, p.K, p.M, lda * eb, 128);
  if (e != cudaSuccess) return e;
  e = make_kmajor_map(&mb, b, eb, p.K, p.N, ldb * eb, bn);
  if (e != cudaSuccess) return e;
  p.tiles_m = static_cast<int>((p.M + 127) / 128);
  const int kb_elems = 128 / eb;
  p.num_kb = static_cast<int>((p.K + kb_elems - 1) / kb_elems);
  if (kind == kKindI8)
    return bn == 256 ? launch_gemm<kKindI8, 256, 4>(ma, mb, p, max_ctas, stream)
                     : launch_gemm<kKindI8, 128, 6>(ma, mb, p, max_ctas, stream);
  if (kind == kKindE4M3)
    return bn == 256 ? launch_gemm<kKindE4M3, 256, 4>(ma, mb, p, max_ctas, stream)
                     : launch_gemm<kKindE4M3, 128, 6>(ma, mb, p, max_ctas, stream);
  return bn == 256 ? launch_gemm<kKindBF16, 256, 4>(ma, mb, p, max_ctas, stream)
                   : launch_gemm<kKindBF16, 128, 6>(ma, mb, p, max_ctas, stream);
}

}  // namespace b2

// Synchronous read of the device status word (see include/b2_qlinear.h).
extern "C" int b2_device_status(int* status, int reset) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, b2::g_b2_status, sizeof(int));
  if (e != cudaSuccess) return static_cast<int>(e);
  if (status) *status = v;
  if (reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(b2::g_b2_status, &zero, sizeof(int));
  }
  return static_cast<int>(e);
}
