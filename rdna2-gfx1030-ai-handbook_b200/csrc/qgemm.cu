// Quantized GEMM with fused dequant epilogue for sm_100a.
//
// C[m,n] = epilogue( sum_k A[m,k] * B[n,k] )  with A [M,K] and B [N,K] both
// K-major (B is the weight in its stored [N,K] layout, i.e. the reference's
// `weight.T` view of rdna2_ops/int8_gemm.py:39-40 without a copy).
//
// Two persistent, warp-specialized kernels (192 threads per CTA, one CTA per
// SM):
//   qgemm_pair_kernel  2-CTA cluster; the leader CTA issues tcgen05.mma
//                      .cta_group::2 on a 256 x BN tile whose A rows and B
//                      columns are split across the two CTAs' shared memory,
//                      so each SM reads half the B operand per MMA and the
//                      ring holds 6-7 stages.  Used whenever M > 128.
//   qgemm_kernel       single CTA, 128 x BN tile; small-M problems.
// Roles in both:
//   warp 0      TMA producer into a STAGES-deep ring of 128B-swizzled k-blocks
//               (plain tile loads; pair loads count bytes on the leader's
//               barrier; never multicast).
//   warp 1      TMEM owner + single-thread MMA issuer (kind::i8 for W8A8,
//               kind::f8f6f4 for e4m3, kind::f16 for bf16), 4 MMAs of 32 bytes
//               of K per k-block; commits free ring slots and publish finished
//               accumulators.
//   warps 2..5  epilogue: double-buffered TMEM accumulators let tile t+1's
//               MMAs overlap tile t's epilogue; tcgen05.ld ping-pong buffers,
//               per-token x per-channel scale, bias and cast; the pair
//               kernel stages each 32-row x 128-byte unit in swizzled shared
//               memory and writes it with a TMA store (6-stage ring), or,
//               for unaligned outputs, stores 16 bytes per lane (7 stages).
//
// Epilogue rounding follows the reference exactly:
//   separate  float(acc)*(sa*sb) then + bias in fp32, two roundings
//             (rdna2_ops/int8_gemm.py:53-63 with enable_fp_fusion=False)
//   fma       fma(float(acc), sa*sb, bias)       (rounding="fused", :191)
//   kitchen   (float(acc)*(sa*sb)).to(out) + bias.to(out)
//             (production/MOSS_RDNA2_INT8/backend.py:128-143)
//   none      raw INT32 accumulator              (int8_matmul, :195-200)
#include <cstring>
#include <mutex>

#include "b2_common.cuh"
#include "b2_internal.h"

namespace b2 {

__device__ int g_b2_status = 0;

int* status_word_ptr() {
  static int* cache[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_b2_status) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    cache[dev] = static_cast<int*>(p);
  }
  return cache[dev];
}

constexpr int kEpiWarps = 4;

__host__ __device__ constexpr uint32_t tmem_cols_for(int cols) {
  return cols <= 32 ? 32 : cols <= 64 ? 64 : cols <= 128 ? 128 : cols <= 256 ? 256 : 512;
}

// Output staging of the TMA-store epilogue: per epilogue warp, two 4 KiB
// buffers of 32 rows x 128 bytes (128-byte swizzled, the layout the store's
// tensor map reads).
constexpr int kOutBufBytes = 32 * 128;
constexpr int kOutStageBytes = kEpiWarps * 2 * kOutBufBytes;

// Shared-memory plan: A ring, B ring, optional output staging, per-warp
// staging of one 32-column chunk of epilogue scale/bias, barriers.
template <int A_ROWS, int B_ROWS, int BN, int STAGES, int OUT_STAGE = 0>
struct Smem {
  static constexpr int kABytes = A_ROWS * 128;
  static constexpr int kBBytes = B_ROWS * 128;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kOffA = 0;
  static constexpr int kOffB = STAGES * kABytes;
  static constexpr int kOffOut = STAGES * kStageBytes;  // 1 KiB aligned (stage sizes are)
  static constexpr int kOffEpi = kOffOut + OUT_STAGE;
  static constexpr int kOffBar = kOffEpi + kEpiWarps * 64 * 4;
  static constexpr int kNumBars = 2 * STAGES + 4;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kBytes = kOffMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
  static constexpr uint32_t kTmemCols = tmem_cols_for(2 * BN);
  static_assert(kABytes % 1024 == 0 && kBBytes % 1024 == 0, "swizzle atoms need 1 KiB alignment");
  static_assert(kAlloc <= 232448, "shared memory budget");
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

// Epilogue values of one thread's 32 accumulator columns; the chunk's
// per-channel scales and bias come from this warp's shared staging.
template <int KIND, int MODE, int OUT>
__device__ __forceinline__ void chunk_values(const GemmParams& p, const uint32_t (&r)[32], float sa,
                                             const float* csb, const float* cbias, float (&v)[32]) {
  const bool hb = p.bias != nullptr;
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    const float4 s4 = *reinterpret_cast<const float4*>(csb + j);
    const float4 b4 = *reinterpret_cast<const float4*>(cbias + j);
    const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
    const float bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (MODE == kEpiNone) {
        v[j + i] = __uint_as_float(r[j + i]);
      } else {
        v[j + i] = epi_value<KIND, MODE, OUT>(r[j + i], sa, sv[i], bv[i], hb);
      }
    }
  }
}

// One thread, one output row, 32 consecutive columns starting at n, stored
// straight to global memory.
template <int KIND, int MODE, int OUT>
__device__ __forceinline__ void store_chunk(const GemmParams& p, const uint32_t (&r)[32], int row,
                                            int n, float sa, const float* csb, const float* cbias) {
  if (row >= p.M) return;
  float v[32];
  chunk_values<KIND, MODE, OUT>(p, r, sa, csb, cbias, v);
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
                                               int n, float sa, const float* csb, const float* cb) {
  switch (p.epilogue * 4 + p.out_dtype) {
    case kEpiNone * 4 + kI32: store_chunk<KIND, kEpiNone, kI32>(p, r, row, n, sa, csb, cb); break;
    case kEpiSeparate * 4 + kF32: store_chunk<KIND, kEpiSeparate, kF32>(p, r, row, n, sa, csb, cb); break;
    case kEpiSeparate * 4 + kF16: store_chunk<KIND, kEpiSeparate, kF16>(p, r, row, n, sa, csb, cb); break;
    case kEpiSeparate * 4 + kBF16: store_chunk<KIND, kEpiSeparate, kBF16>(p, r, row, n, sa, csb, cb); break;
    case kEpiFma * 4 + kF32: store_chunk<KIND, kEpiFma, kF32>(p, r, row, n, sa, csb, cb); break;
    case kEpiFma * 4 + kF16: store_chunk<KIND, kEpiFma, kF16>(p, r, row, n, sa, csb, cb); break;
    case kEpiFma * 4 + kBF16: store_chunk<KIND, kEpiFma, kBF16>(p, r, row, n, sa, csb, cb); break;
    case kEpiKitchen * 4 + kF32: store_chunk<KIND, kEpiKitchen, kF32>(p, r, row, n, sa, csb, cb); break;
    case kEpiKitchen * 4 + kF16: store_chunk<KIND, kEpiKitchen, kF16>(p, r, row, n, sa, csb, cb); break;
    case kEpiKitchen * 4 + kBF16: store_chunk<KIND, kEpiKitchen, kBF16>(p, r, row, n, sa, csb, cb); break;
    default: break;
  }
}

// One thread, one staging row (32 rows x 128 bytes, 128-byte swizzle: the
// 16-byte piece j of row r sits at piece j ^ (r % 8)), 32 columns written at
// piece offset piece0 (16-bit outputs fill a row with two chunks, 32-bit
// outputs with one).  The swizzle keeps each quarter-warp's 16-byte stores on
// distinct banks.
template <int KIND, int MODE, int OUT>
__device__ __forceinline__ void stage_chunk(const GemmParams& p, const uint32_t (&r)[32], uint32_t row_addr,
                                            int lane, int piece0, float sa, const float* csb,
                                            const float* cbias) {
  float v[32];
  chunk_values<KIND, MODE, OUT>(p, r, sa, csb, cbias, v);
  const uint32_t sw = static_cast<uint32_t>(lane & 7);
  if constexpr (OUT == kF32 || OUT == kI32) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      sts_v4(row_addr + ((static_cast<uint32_t>(j + piece0) ^ sw) << 4),
             make_uint4(__float_as_uint(v[4 * j]), __float_as_uint(v[4 * j + 1]),
                        __float_as_uint(v[4 * j + 2]), __float_as_uint(v[4 * j + 3])));
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      sts_v4(row_addr + ((static_cast<uint32_t>(j + piece0) ^ sw) << 4),
             make_uint4(pack2(v[8 * j], v[8 * j + 1], OUT), pack2(v[8 * j + 2], v[8 * j + 3], OUT),
                        pack2(v[8 * j + 4], v[8 * j + 5], OUT), pack2(v[8 * j + 6], v[8 * j + 7], OUT)));
  }
}

template <int KIND>
__device__ __forceinline__ void stage_dispatch(const GemmParams& p, const uint32_t (&r)[32], uint32_t row_addr,
                                               int lane, int piece0, float sa, const float* csb,
                                               const float* cb) {
  switch (p.epilogue * 4 + p.out_dtype) {
    case kEpiNone * 4 + kI32: stage_chunk<KIND, kEpiNone, kI32>(p, r, row_addr, lane, piece0, sa, csb, cb); break;
    case kEpiSeparate * 4 + kF32: stage_chunk<KIND, kEpiSeparate, kF32>(p, r, row_addr, lane, piece0, sa, csb, cb); break;
    case kEpiSeparate * 4 + kF16: stage_chunk<KIND, kEpiSeparate, kF16>(p, r, row_addr, lane, piece0, sa, csb, cb); break;
    case kEpiSeparate * 4 + kBF16: stage_chunk<KIND, kEpiSeparate, kBF16>(p, r, row_addr, lane, piece0, sa, csb, cb); break;
    case kEpiFma * 4 + kF32: stage_chunk<KIND, kEpiFma, kF32>(p, r, row_addr, lane, piece0, sa, csb, cb); break;
    case kEpiFma * 4 + kF16: stage_chunk<KIND, kEpiFma, kF16>(p, r, row_addr, lane, piece0, sa, csb, cb); break;
    case kEpiFma * 4 + kBF16: stage_chunk<KIND, kEpiFma, kBF16>(p, r, row_addr, lane, piece0, sa, csb, cb); break;
    case kEpiKitchen * 4 + kF32: stage_chunk<KIND, kEpiKitchen, kF32>(p, r, row_addr, lane, piece0, sa, csb, cb); break;
    case kEpiKitchen * 4 + kF16: stage_chunk<KIND, kEpiKitchen, kF16>(p, r, row_addr, lane, piece0, sa, csb, cb); break;
    case kEpiKitchen * 4 + kBF16: stage_chunk<KIND, kEpiKitchen, kBF16>(p, r, row_addr, lane, piece0, sa, csb, cb); break;
    default: break;
  }
}

// Per-lane scale and bias of column n (Kitchen mode pre-rounds the bias
// through the output dtype, as `bias.to(out_dtype)` does).
__device__ __forceinline__ void load_col(const GemmParams& p, int n, float sb0, float& sb, float& b) {
  sb = sb0;
  b = 0.0f;
  if (n < p.N) {
    if (p.sb != nullptr && !p.sb_scalar) sb = p.sb[n];
    if (p.bias != nullptr) {
      b = load_as_float(p.bias, p.bias_dtype, n);
      if (p.epilogue == kEpiKitchen) {
        if (p.out_dtype == kF16) b = round_through<kF16>(b);
        if (p.out_dtype == kBF16) b = round_through<kBF16>(b);
      }
    }
  }
}

// Epilogue of one accumulator tile by one warp (32 rows x BN columns), one
// 32-column chunk at a time.  TMEM loads are double buffered (chunk c+1 in
// flight while chunk c is converted and stored) and the next chunk's scale
// and bias are fetched into registers while the current chunk is stored.
// `release` runs once every TMEM read of the tile has completed.
template <int KIND, int BN, typename Release>
__device__ __forceinline__ void epilogue_tile(const GemmParams& p, uint32_t taddr, int row, int n0,
                                              int lane, float* wst, Release release) {
  constexpr int NC = BN / 32;
  static_assert(NC % 2 == 0, "ping-pong over chunk pairs");
  const float sb0 = (p.sb != nullptr && p.sb_scalar) ? p.sb[0] : 0.0f;
  const float sa = (p.sa != nullptr && row < p.M) ? p.sa[row] : 0.0f;
  float sb_n, b_n;
  load_col(p, n0 + lane, sb0, sb_n, b_n);
  uint32_t r0[32], r1[32];
  __syncwarp();
  tmem_ld32(taddr, r0);
  tmem_ld_wait(r0);
#pragma unroll 1
  for (int c = 0; c < NC; c += 2) {
    // chunk c (in r0)
    __syncwarp();
    wst[lane] = sb_n;
    wst[32 + lane] = b_n;
    __syncwarp();
    load_col(p, n0 + (c + 1) * 32 + lane, sb0, sb_n, b_n);
    tmem_ld32(taddr + static_cast<uint32_t>((c + 1) * 32), r1);
    store_dispatch<KIND>(p, r0, row, n0 + c * 32, sa, wst, wst + 32);
    __syncwarp();
    tmem_ld_wait(r1);
    if (c + 2 < NC) {
      tmem_ld32(taddr + static_cast<uint32_t>((c + 2) * 32), r0);
    } else {
      release();  // all TMEM reads of this tile are complete
    }
    // chunk c+1 (in r1)
    __syncwarp();
    wst[lane] = sb_n;
    wst[32 + lane] = b_n;
    __syncwarp();
    if (c + 2 < NC) load_col(p, n0 + (c + 2) * 32 + lane, sb0, sb_n, b_n);
    store_dispatch<KIND>(p, r1, row, n0 + (c + 1) * 32, sa, wst, wst + 32);
    __syncwarp();
    if (c + 2 < NC) tmem_ld_wait(r0);
  }
}

// Tensor maps of the peers' outputs (same geometry as this rank's output
// map, other base addresses), a kernel parameter of the gather kernels only.
template <bool GATHER>
struct PeerMaps {
  CUtensorMap m[kMaxGatherPeers];
};
template <>
struct PeerMaps<false> {
  int unused;
};

// Column-parallel gather: copy one staged unit (32 rows x 128 bytes at
// `buf`, 128-byte swizzle) to every peer output with 16-byte stores, four
// whole 128-byte row segments per warp instruction.  Gather mode requires
// N % 64 == 0 and 16-byte aligned output rows, so a piece is either wholly
// inside the output or wholly past it.
__device__ __forceinline__ void peer_store_unit(const GemmParams& p, uint32_t buf, int row0, int x, int lane) {
  const int ob = (p.out_dtype == kF16 || p.out_dtype == kBF16) ? 2 : 4;
  const int j = lane & 7;
  if (x + j * (16 / ob) >= p.N) return;
#pragma unroll 2
  for (int i = 0; i < 8; ++i) {
    const int r = i * 4 + (lane >> 3);
    const uint4 v = lds_v4(buf + static_cast<uint32_t>(r * 128) + (static_cast<uint32_t>(j ^ (r & 7)) << 4));
    if (row0 + r < p.M) {
      const int64_t off = (static_cast<int64_t>(row0 + r) * p.ldc + x) * ob + j * 16;
      for (int q = 0; q < p.n_peers; ++q) st_global_v4(static_cast<char*>(p.peer_out[q]) + off, v);
    }
  }
}

// End of a gather-mode kernel, run by all epilogue threads of every CTA:
// each orders its peer stores before a CTA-wide barrier with a system-scope
// fence; one thread per CTA counts the CTA; the last CTA fences again and
// releases `epoch` into every flag slot (the peers' arrays and its own), then
// rearms the counter for the next launch on the stream.
constexpr int kGatherBarrier = 2;

__device__ __forceinline__ void gather_signal(const GemmParams& p) {
  __threadfence_system();
  named_bar_sync(kGatherBarrier, kEpiWarps * 32);
  if (threadIdx.x == 64) {  // first epilogue thread
    const uint32_t prev = atomicAdd(p.done_count, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      for (int q = 0; q <= p.n_peers; ++q) st_release_sys(p.flag_slot[q], p.epoch);
      *p.done_count = 0u;
    }
  }
}

// The same epilogue with the output staged through shared memory: each
// 128-byte-wide column unit of the warp's 32 rows is written into one of two
// swizzled staging buffers and leaves as one TMA store (whole 128-byte lines
// to L2 instead of 32 half-sector stores per instruction), while the next
// unit is converted.  Lane 0 issues and waits on the warp's bulk groups; the
// tensor map clips rows >= M and columns >= N.
template <int KIND, int BN, bool GATHER, typename Release>
__device__ __forceinline__ void epilogue_tile_tma(const GemmParams& p, const CUtensorMap* tma_c,
                                                  const PeerMaps<GATHER>* pm, uint32_t taddr, int row, int row0,
                                                  int n0, int lane, float* wst, uint32_t obuf, uint32_t& ob_sel,
                                                  Release release) {
  constexpr int NC = BN / 32;
  static_assert(NC % 2 == 0, "ping-pong over chunk pairs");
  const int uc = (p.out_dtype == kF16 || p.out_dtype == kBF16) ? 2 : 1;  // chunks per staging row
  const float sb0 = (p.sb != nullptr && p.sb_scalar) ? p.sb[0] : 0.0f;
  const float sa = (p.sa != nullptr && row < p.M) ? p.sa[row] : 0.0f;
  auto emit = [&](const uint32_t (&r)[32], int c) {
    const int part = c & (uc - 1);
    if (part == 0) {
      if (lane == 0) bulk_wait_read<1>();  // the buffer's previous store has read it
      __syncwarp();
    }
    const uint32_t buf = obuf + ob_sel * static_cast<uint32_t>(kOutBufBytes);
    stage_dispatch<KIND>(p, r, buf + static_cast<uint32_t>(lane) * 128u, lane, part * 4, sa, wst, wst + 32);
    if (part == uc - 1) {
      fence_proxy_async_smem();  // generic-proxy writes visible to the TMA
      __syncwarp();
      const int x = n0 + (c - part) * 32;
      if (lane == 0 && row0 < p.M && x < p.N) {
        tma_store_2d(tma_c, buf, x, row0);
        if constexpr (GATHER) {
          if (p.gather == kGatherTma)
            for (int q = 0; q < p.n_peers; ++q) tma_store_2d(&pm->m[q], buf, x, row0);
        }
        bulk_commit_group();
      }
      if constexpr (GATHER) {
        if (p.gather != kGatherTma) peer_store_unit(p, buf, row0, x, lane);
      }
      ob_sel ^= 1u;
    }
  };
  float sb_n, b_n;
  load_col(p, n0 + lane, sb0, sb_n, b_n);
  uint32_t r0[32], r1[32];
  __syncwarp();
  tmem_ld32(taddr, r0);
  tmem_ld_wait(r0);
#pragma unroll 1
  for (int c = 0; c < NC; c += 2) {
    __syncwarp();
    wst[lane] = sb_n;
    wst[32 + lane] = b_n;
    __syncwarp();
    load_col(p, n0 + (c + 1) * 32 + lane, sb0, sb_n, b_n);
    tmem_ld32(taddr + static_cast<uint32_t>((c + 1) * 32), r1);
    emit(r0, c);
    __syncwarp();
    tmem_ld_wait(r1);
    if (c + 2 < NC) {
      tmem_ld32(taddr + static_cast<uint32_t>((c + 2) * 32), r0);
    } else {
      release();  // all TMEM reads of this tile are complete
    }
    __syncwarp();
    wst[lane] = sb_n;
    wst[32 + lane] = b_n;
    __syncwarp();
    if (c + 2 < NC) load_col(p, n0 + (c + 2) * 32 + lane, sb0, sb_n, b_n);
    emit(r1, c + 1);
    __syncwarp();
    if (c + 2 < NC) tmem_ld_wait(r0);
  }
}

// --------------------------------------------------------- 1-CTA kernel
template <int KIND, int BN, int STAGES>
__global__ void __launch_bounds__(192, 1)
    qgemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                 const GemmParams p) {
  using L = Smem<128, BN, BN, STAGES>;
  constexpr int kKbElems = (KIND == kKindBF16 || KIND == kKindF16) ? 64 : 128;  // 128 bytes of K per k-block
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
      mbar_init(&tempty[b], kEpiWarps);
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
    // Producer.  The whole warp runs the loop and one elected lane issues:
    // a loop run by a single lane of a diverged warp pays a large
    // per-iteration cost on this part.
    griddep_wait();  // operands may come from the previous kernel
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      const int tm = tile % p.tiles_m, tn = tile / p.tiles_m;
      for (int kb = 0; kb < p.num_kb; ++kb) {
        ok = __all_sync(0xffffffffu, mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kSiteProducer, p.status));
        if (!ok) break;
        if (elect_one()) {
          mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
          tma_load_2d(&tma_a, &full[stage], smem + L::kOffA + stage * L::kABytes, kb * kKbElems, tm * 128);
          tma_load_2d(&tma_b, &full[stage], smem + L::kOffB + stage * L::kBBytes, kb * kKbElems, tn * BN);
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    // Tail: wait until the MMA warp has released every slot, so no commit
    // is still in flight to this CTA's barriers when it exits.
    for (int i = 0; i < STAGES && ok; ++i) {
      ok = __all_sync(0xffffffffu, mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kSiteProducer, p.status));
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
  } else if (warp == 1) {
    // MMA issuer: whole warp loops, one elected lane (the same lane every
    // time, so its commits cover its own MMAs) issues.  Descriptors are
    // built once; stepping stages and K slices adds to the address field.
    constexpr uint32_t idesc = make_idesc<KIND>(128, BN);
    const uint64_t a_desc0 = sw128_desc(smem_u32(smem + L::kOffA));
    const uint64_t b_desc0 = sw128_desc(smem_u32(smem + L::kOffB));
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    int t = 0;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++t) {
      const int buf = t & 1;
      const uint32_t use = static_cast<uint32_t>(t >> 1);
      ok = __all_sync(0xffffffffu, mbar_wait(&tempty[buf], (use & 1u) ^ 1u, abort_flag, kSiteMmaTmem, p.status));
      if (!ok) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * BN);
      for (int kb = 0; kb < p.num_kb; ++kb) {
        ok = __all_sync(0xffffffffu, mbar_wait(&full[stage], phase, abort_flag, kSiteMma, p.status));
        if (!ok) break;
        tc_fence_after();
        if (elect_one()) {
          const uint64_t ad = a_desc0 + static_cast<uint32_t>((stage * L::kABytes) >> 4);
          const uint64_t bd = b_desc0 + static_cast<uint32_t>((stage * L::kBBytes) >> 4);
          umma<KIND>(d_tmem, ad, bd, idesc, kb != 0 ? 1u : 0u);
          umma<KIND>(d_tmem, ad + 2, bd + 2, idesc, 1u);
          umma<KIND>(d_tmem, ad + 4, bd + 4, idesc, 1u);
          umma<KIND>(d_tmem, ad + 6, bd + 6, idesc, 1u);
          umma_commit(&empty[stage]);
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      if (elect_one()) umma_commit(&tfull[buf]);
      __syncwarp();
    }
  } else {
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    float* wsb = reinterpret_cast<float*>(smem + L::kOffEpi) + (warp - 2) * 64;
    griddep_wait();
    int t = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++t) {
      const int buf = t & 1;
      const uint32_t use = static_cast<uint32_t>(t >> 1);
      const int tm = tile % p.tiles_m, tn = tile / p.tiles_m;
      bool ok = mbar_wait(&tfull[buf], use & 1u, abort_flag, kSiteEpilogue, p.status);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(buf * BN);
      epilogue_tile<KIND, BN>(p, taddr, tm * 128 + quarter * 32 + lane, tn * BN, lane, wsb, [&] {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[buf]);
      });
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// ------------------------------------------------------- 2-CTA kernel
// Cluster of two CTAs computes a 256 x BN tile: CTA r holds A rows
// [128r, 128r+128) and B rows [r*BN/2, (r+1)*BN/2) of every k-block and
// accumulates its 128 x BN half in its own TMEM.  The leader (rank 0) waits
// on its `full` barrier (both CTAs' loads count there), issues the pair MMAs
// and signals both CTAs' `empty` / `tfull` barriers with one commit each;
// both epilogues hand TMEM back through the leader's `tempty` barrier (8
// arrivals).
template <int KIND, int BN, int STAGES, bool TSTORE, bool GATHER = false>
__global__ void __launch_bounds__(192, 1)
    qgemm_pair_kernel(const __grid_constant__ CUtensorMap tma_a,
                      const __grid_constant__ CUtensorMap tma_b,
                      const __grid_constant__ CUtensorMap tma_c,
                      const __grid_constant__ PeerMaps<GATHER> peer_maps, const GemmParams p) {
  using L = Smem<128, BN / 2, BN, STAGES, TSTORE ? kOutStageBytes : 0>;
  constexpr int kKbElems = (KIND == kKindBF16 || KIND == kKindF16) ? 64 : 128;
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
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(cluster_id_x());
  const int npairs = static_cast<int>(cluster_count_x());
  const int num_tiles = p.tiles_m * p.tiles_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * kEpiWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, L::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // Producer (whole warp loops, one elected lane issues).
    griddep_wait();  // operands may come from the previous kernel
    const uint32_t full_leader = mapa_shared(smem_u32(&full[0]), 0);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int tile = pair; tile < num_tiles && ok; tile += npairs) {
      const int tm = tile % p.tiles_m, tn = tile / p.tiles_m;
      for (int kb = 0; kb < p.num_kb; ++kb) {
        ok = __all_sync(0xffffffffu, mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kSiteProducer, p.status));
        if (!ok) break;
        if (elect_one()) {
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * L::kStageBytes);
          const uint32_t fb = full_leader + static_cast<uint32_t>(stage * 8);
          tma_load_2d_pair(&tma_a, fb, smem + L::kOffA + stage * L::kABytes, kb * kKbElems,
                           tm * 256 + static_cast<int>(rank) * 128);
          tma_load_2d_pair(&tma_b, fb, smem + L::kOffB + stage * L::kBBytes, kb * kKbElems,
                           tn * BN + static_cast<int>(rank) * (BN / 2));
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    // Tail: every slot released before exit.
    for (int i = 0; i < STAGES && ok; ++i) {
      ok = __all_sync(0xffffffffu, mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kSiteProducer, p.status));
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
  } else if (warp == 1) {
    if (leader) {
      // MMA issuer of the pair (leader CTA): whole warp loops, one elected
      // lane issues; descriptors built once, stages stepped by adds.
      constexpr uint32_t idesc = make_idesc<KIND>(256, BN);
      const uint64_t a_desc0 = sw128_desc(smem_u32(smem + L::kOffA));
      const uint64_t b_desc0 = sw128_desc(smem_u32(smem + L::kOffB));
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int t = 0;
      for (int tile = pair; tile < num_tiles && ok; tile += npairs, ++t) {
        const int buf = t & 1;
        const uint32_t use = static_cast<uint32_t>(t >> 1);
        ok = __all_sync(0xffffffffu,
                        mbar_wait(&tempty[buf], (use & 1u) ^ 1u, abort_flag, kSiteMmaTmem, p.status));
        if (!ok) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * BN);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          ok = __all_sync(0xffffffffu, mbar_wait(&full[stage], phase, abort_flag, kSiteMma, p.status));
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            const uint64_t ad = a_desc0 + static_cast<uint32_t>((stage * L::kABytes) >> 4);
            const uint64_t bd = b_desc0 + static_cast<uint32_t>((stage * L::kBBytes) >> 4);
            umma_pair<KIND>(d_tmem, ad, bd, idesc, kb != 0 ? 1u : 0u);
            umma_pair<KIND>(d_tmem, ad + 2, bd + 2, idesc, 1u);
            umma_pair<KIND>(d_tmem, ad + 4, bd + 4, idesc, 1u);
            umma_pair<KIND>(d_tmem, ad + 6, bd + 6, idesc, 1u);
            // One completion signal to both CTAs' `empty[stage]` barriers.
            umma_commit_pair_both(smem_u32(&empty[stage]));
          }
          __syncwarp();
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (elect_one()) umma_commit_pair_both(smem_u32(&tfull[buf]));
        __syncwarp();
      }
    }
  } else {
    const int quarter = warp & 3;
    float* wsb = reinterpret_cast<float*>(smem + L::kOffEpi) + (warp - 2) * 64;
    const uint32_t tempty_leader = mapa_shared(smem_u32(&tempty[0]), 0);
    const uint32_t obuf = smem_u32(smem + L::kOffOut) + static_cast<uint32_t>((warp - 2) * 2 * kOutBufBytes);
    uint32_t ob_sel = 0;
    griddep_wait();
    int t = 0;
    for (int tile = pair; tile < num_tiles; tile += npairs, ++t) {
      const int buf = t & 1;
      const uint32_t use = static_cast<uint32_t>(t >> 1);
      const int tm = tile % p.tiles_m, tn = tile / p.tiles_m;
      bool ok = mbar_wait(&tfull[buf], use & 1u, abort_flag, kSiteEpilogue, p.status);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(buf * BN);
      const int row0 = tm * 256 + static_cast<int>(rank) * 128 + quarter * 32;
      auto release = [&] {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(tempty_leader + static_cast<uint32_t>(buf * 8));
      };
      if constexpr (TSTORE) {
        epilogue_tile_tma<KIND, BN, GATHER>(p, &tma_c, &peer_maps, taddr, row0 + lane, row0, tn * BN, lane, wsb,
                                            obuf, ob_sel, release);
      } else {
        epilogue_tile<KIND, BN>(p, taddr, row0 + lane, tn * BN, lane, wsb, release);
      }
    }
    if constexpr (TSTORE) {
      if (lane == 0) {
        bulk_wait_all();  // staging reads and global writes (this GPU's and the peers') done
        if constexpr (GATHER) fence_proxy_async_global();
      }
      __syncwarp();
    }
    if constexpr (GATHER) gather_signal(p);
  }

  tc_fence_before();
  cluster_sync();  // no CTA leaves while its peer may still touch its barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, L::kTmemCols);
  }
}

// ------------------------------------------------ split-K kernel (M <= 32)
// Decode-sized problems (M <= 32 tokens) are weight-streaming bound: with
// 128 x BN output tiles only ceil(N/128) SMs would read the weights.  Here
// the weight tile is the 128-row A operand and the tokens the N = BT
// operand (swap-AB), and each 128-row tile is split along K over the S CTAs
// of one thread-block cluster (S <= 8, S * tiles <= SMs).  Every CTA streams
// its contiguous k-block range through a TMA ring into its own TMEM
// accumulator; the S-1 non-leader CTAs then write their accumulators into
// the leader's shared memory over distributed shared memory, and after one
// cluster barrier the leader adds them in rank order (exact for int32,
// a fixed order for fp32) and runs the epilogue.  No global workspace, no
// inter-CTA spin waits.
constexpr int kSplitMax = 8;

template <int BT, int STAGES>
struct SplitSmem {
  static constexpr int kWBytes = 128 * 128;
  static constexpr int kXBytes = BT * 128;
  static constexpr int kStageBytes = kWBytes + kXBytes;
  static constexpr int kOffW = 0;
  static constexpr int kOffX = STAGES * kWBytes;
  static constexpr int kOffPart = kOffX + STAGES * kXBytes;              // [S-1][128][BT] 32-bit
  static constexpr int kOffBar = kOffPart + (kSplitMax - 1) * 128 * BT * 4;
  static constexpr int kOffMisc = kOffBar + (2 * STAGES + 1) * 8;
  static constexpr int kBytes = kOffMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;
  static_assert(kXBytes % 1024 == 0, "swizzle atoms need 1 KiB alignment");
  static_assert(kAlloc <= 232448, "shared memory budget");
};

template <int KIND, int MODE, int OUT, int BT>
__device__ __forceinline__ void splitk_store(const GemmParams& p, const uint32_t (&v)[BT], int n) {
  if (n >= p.N) return;
  float sb = 0.0f, b = 0.0f;
  load_col(p, n, (p.sb != nullptr && p.sb_scalar) ? p.sb[0] : 0.0f, sb, b);
  const bool hb = p.bias != nullptr;
  const int mt = p.M < BT ? p.M : BT;
#pragma unroll
  for (int t = 0; t < BT; ++t) {
    if (t >= mt) break;
    float y;
    if constexpr (MODE == kEpiNone) {
      y = __uint_as_float(v[t]);
    } else {
      y = epi_value<KIND, MODE, OUT>(v[t], p.sa[t], sb, b, hb);
    }
    const int64_t o = static_cast<int64_t>(t) * p.ldc + n;
    if constexpr (OUT == kF32 || OUT == kI32) {
      static_cast<uint32_t*>(p.out)[o] = __float_as_uint(y);
    } else if constexpr (OUT == kF16) {
      static_cast<__half*>(p.out)[o] = __float2half_rn(y);
    } else {
      static_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16_rn(y);
    }
  }
}

template <int KIND, int BT>
__device__ __forceinline__ void splitk_store_dispatch(const GemmParams& p, const uint32_t (&v)[BT], int n) {
  switch (p.epilogue * 4 + p.out_dtype) {
    case kEpiNone * 4 + kI32: splitk_store<KIND, kEpiNone, kI32, BT>(p, v, n); break;
    case kEpiSeparate * 4 + kF32: splitk_store<KIND, kEpiSeparate, kF32, BT>(p, v, n); break;
    case kEpiSeparate * 4 + kF16: splitk_store<KIND, kEpiSeparate, kF16, BT>(p, v, n); break;
    case kEpiSeparate * 4 + kBF16: splitk_store<KIND, kEpiSeparate, kBF16, BT>(p, v, n); break;
    case kEpiFma * 4 + kF32: splitk_store<KIND, kEpiFma, kF32, BT>(p, v, n); break;
    case kEpiFma * 4 + kF16: splitk_store<KIND, kEpiFma, kF16, BT>(p, v, n); break;
    case kEpiFma * 4 + kBF16: splitk_store<KIND, kEpiFma, kBF16, BT>(p, v, n); break;
    case kEpiKitchen * 4 + kF32: splitk_store<KIND, kEpiKitchen, kF32, BT>(p, v, n); break;
    case kEpiKitchen * 4 + kF16: splitk_store<KIND, kEpiKitchen, kF16, BT>(p, v, n); break;
    case kEpiKitchen * 4 + kBF16: splitk_store<KIND, kEpiKitchen, kBF16, BT>(p, v, n); break;
    default: break;
  }
}

template <int KIND, int BT, int STAGES>
__global__ void __launch_bounds__(192, 1)
    qgemm_splitk_kernel(const __grid_constant__ CUtensorMap tma_w, const __grid_constant__ CUtensorMap tma_x,
                        const GemmParams p) {
  using L = SplitSmem<BT, STAGES>;
  constexpr int kKbElems = (KIND == kKindBF16 || KIND == kKindF16) ? 64 : 128;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = static_cast<int>(cluster_ctarank());
  const int splits = static_cast<int>(gridDim.x) / p.tiles_m;  // cluster size
  const int tile = static_cast<int>(cluster_id_x());
  const int kb0 = static_cast<int>((static_cast<int64_t>(rank) * p.num_kb) / splits);
  const int kb1 = static_cast<int>((static_cast<int64_t>(rank + 1) * p.num_kb) / splits);
  constexpr uint32_t kTmemCols = tmem_cols_for(BT);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tma_w);
    tma_prefetch_desc(&tma_x);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  cluster_sync();  // every CTA of the cluster running, barriers and TMEM ready
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // Inside the fused linear the weights do not depend on the previous
    // kernel (its activation prologue): the first ring's worth streams in
    // before the wait.  Other callers wait first (p.weight_prefetch == 0).
    const int pre = kb1 - kb0 < STAGES ? kb1 - kb0 : STAGES;
    if (!p.weight_prefetch) griddep_wait();
    if (elect_one()) {
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], L::kStageBytes);
        tma_load_2d(&tma_w, &full[i], smem + L::kOffW + i * L::kWBytes, (kb0 + i) * kKbElems, tile * 128);
      }
    }
    __syncwarp();
    if (p.weight_prefetch) griddep_wait();
    if (elect_one()) {
      for (int i = 0; i < pre; ++i)
        tma_load_2d(&tma_x, &full[i], smem + L::kOffX + i * L::kXBytes, (kb0 + i) * kKbElems, 0);
    }
    __syncwarp();
    int stage = pre == STAGES ? 0 : pre;
    uint32_t phase = pre == STAGES ? 1u : 0u;
    bool ok = true;
    for (int kb = kb0 + pre; kb < kb1 && ok; ++kb) {
      ok = __all_sync(0xffffffffu, mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kSiteProducer, p.status));
      if (!ok) break;
      if (elect_one()) {
        mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
        tma_load_2d(&tma_w, &full[stage], smem + L::kOffW + stage * L::kWBytes, kb * kKbElems, tile * 128);
        tma_load_2d(&tma_x, &full[stage], smem + L::kOffX + stage * L::kXBytes, kb * kKbElems, 0);
      }
      __syncwarp();
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
    for (int i = 0; i < STAGES && ok; ++i) {  // every slot released before exit
      ok = __all_sync(0xffffffffu, mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kSiteProducer, p.status));
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc = make_idesc<KIND>(128, BT);
    const uint64_t w_desc0 = sw128_desc(smem_u32(smem + L::kOffW));
    const uint64_t x_desc0 = sw128_desc(smem_u32(smem + L::kOffX));
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int kb = kb0; kb < kb1 && ok; ++kb) {
      ok = __all_sync(0xffffffffu, mbar_wait(&full[stage], phase, abort_flag, kSiteMma, p.status));
      if (!ok) break;
      tc_fence_after();
      if (elect_one()) {
        const uint64_t wd = w_desc0 + static_cast<uint32_t>((stage * L::kWBytes) >> 4);
        const uint64_t xd = x_desc0 + static_cast<uint32_t>((stage * L::kXBytes) >> 4);
        umma<KIND>(tmem_base, wd, xd, idesc, kb != kb0 ? 1u : 0u);
        umma<KIND>(tmem_base, wd + 2, xd + 2, idesc, 1u);
        umma<KIND>(tmem_base, wd + 4, xd + 4, idesc, 1u);
        umma<KIND>(tmem_base, wd + 6, xd + 6, idesc, 1u);
        umma_commit(&empty[stage]);
      }
      __syncwarp();
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
    // the accumulator is complete (or, for an empty k range, stays unread)
    if (elect_one()) umma_commit(acc_full);
    __syncwarp();
  }

  // Epilogue warps 2..5: TMEM lane = weight row (tile * 128 + q * 32 + lane),
  // columns = tokens.
  const int quarter = warp & 3;
  const int row_local = quarter * 32 + lane;
  const bool epi = warp >= 2;
  uint32_t v[BT];
  bool have = false;
  if (epi) griddep_wait();  // scales may come from the previous kernel
  if (epi && kb1 > kb0) {
    have = mbar_wait(acc_full, 0, abort_flag, kSiteEpilogue, p.status);
    have = __all_sync(0xffffffffu, have);
    if (have) {
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
      if constexpr (BT == 16) {
        tmem_ld16(taddr, v);
        tmem_ld_wait16(v);
      } else {
        tmem_ld32(taddr, v);
        tmem_ld_wait(v);
      }
    }
  }
  if (!have) {
#pragma unroll
    for (int t = 0; t < BT; ++t) v[t] = 0u;
  }
  if (epi && rank > 0) {
    // this CTA's partial sums -> the leader's [rank-1][row][BT] slot
    const uint32_t dst = mapa_shared(smem_u32(smem + L::kOffPart), 0) +
                         static_cast<uint32_t>(((rank - 1) * 128 + row_local) * BT * 4);
#pragma unroll
    for (int t = 0; t < BT; t += 4)
      asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(dst + t * 4), "r"(v[t]),
                   "r"(v[t + 1]), "r"(v[t + 2]), "r"(v[t + 3])
                   : "memory");
  }
  tc_fence_before();
  cluster_sync();  // partials visible in the leader; no CTA touches TMEM after this
  if (epi && rank == 0) {
    const uint32_t part = smem_u32(smem + L::kOffPart) + static_cast<uint32_t>(row_local * BT * 4);
    for (int r = 1; r < splits; ++r) {
      const uint32_t src = part + static_cast<uint32_t>((r - 1) * 128 * BT * 4);
#pragma unroll
      for (int t = 0; t < BT; t += 4) {
        const uint4 w = lds_v4(src + t * 4);
        const uint32_t o[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if constexpr (KIND == kKindI8) {
            v[t + i] = static_cast<uint32_t>(static_cast<int>(v[t + i]) + static_cast<int>(o[i]));
          } else {
            v[t + i] = __float_as_uint(__fadd_rn(__uint_as_float(v[t + i]), __uint_as_float(o[i])));
          }
        }
      }
    }
    splitk_store_dispatch<KIND, BT>(p, v, tile * 128 + row_local);
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
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

EncodeTiledFn tensor_map_encoder() { return encoder(); }

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

// Output map of the TMA-store epilogue: dims {N, M}, box {128 bytes of
// columns, 32 rows}, 128-byte swizzle (the staging layout).
static cudaError_t make_out_map(CUtensorMap* map, void* ptr, int elem_bytes, int64_t cols, int64_t rows,
                                int64_t row_stride_bytes) {
  EncodeTiledFn fn = encoder();
  if (fn == nullptr) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride_bytes)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / elem_bytes), 32u};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, ptr,
                  dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

static int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

int device_sm_count() {
  const int dev = current_device();
  static int cache[64] = {0};
  if (dev < 64 && cache[dev] > 0) return cache[dev];
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (n <= 0) n = 148;
  if (dev < 64) cache[dev] = n;
  return n;
}

template <typename Kernel>
static cudaError_t configure_once(Kernel kernel, int smem_bytes, bool* done) {
  const int dev = current_device();
  if (dev >= 64) return cudaErrorInvalidDevice;
  if (!done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    if (e != cudaSuccess) return e;
    done[dev] = true;
  }
  return cudaSuccess;
}

template <int KIND, int BN, int STAGES>
static cudaError_t launch_single(const void* a, int64_t lda, const void* b, int64_t ldb, GemmParams p,
                                 int max_ctas, cudaStream_t stream) {
  using L = Smem<128, BN, BN, STAGES>;
  auto kernel = qgemm_kernel<KIND, BN, STAGES>;
  static bool configured[64] = {false};
  cudaError_t e = configure_once(kernel, L::kAlloc, configured);
  if (e != cudaSuccess) return e;
  const int eb = (KIND == kKindBF16 || KIND == kKindF16) ? 2 : 1;
  CUtensorMap ma, mb;
  if ((e = make_kmajor_map(&ma, a, eb, p.K, p.M, lda * eb, 128)) != cudaSuccess) return e;
  if ((e = make_kmajor_map(&mb, b, eb, p.K, p.N, ldb * eb, BN)) != cudaSuccess) return e;
  p.tiles_m = static_cast<int>((p.M + 127) / 128);
  p.tiles_n = static_cast<int>((p.N + BN - 1) / BN);
  const int tiles = p.tiles_m * p.tiles_n;
  int grid = device_sm_count();
  if (max_ctas > 0 && max_ctas < grid) grid = max_ctas;
  if (tiles < grid) grid = tiles;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see griddep_wait
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = L::kAlloc;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kernel, ma, mb, p);
  return e != cudaSuccess ? e : cudaGetLastError();
}

template <int KIND, int BN, int STAGES, bool TSTORE, bool GATHER = false>
static cudaError_t launch_pair(const void* a, int64_t lda, const void* b, int64_t ldb, GemmParams p,
                               int max_ctas, cudaStream_t stream) {
  using L = Smem<128, BN / 2, BN, STAGES, TSTORE ? kOutStageBytes : 0>;
  auto kernel = qgemm_pair_kernel<KIND, BN, STAGES, TSTORE, GATHER>;
  static bool configured[64] = {false};
  static int max_pairs[64] = {0};
  cudaError_t e = configure_once(kernel, L::kAlloc, configured);
  if (e != cudaSuccess) return e;
  const int dev = current_device();
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see griddep_wait
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = L::kAlloc;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (max_pairs[dev] == 0) {
    cfg.gridDim = dim3(2 * (device_sm_count() / 2));
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = -1;
    }
    max_pairs[dev] = n;
  }
  if (max_pairs[dev] < 0) return cudaErrorNotSupported;
  const int eb = (KIND == kKindBF16 || KIND == kKindF16) ? 2 : 1;
  CUtensorMap ma, mb;
  if ((e = make_kmajor_map(&ma, a, eb, p.K, p.M, lda * eb, 128)) != cudaSuccess) return e;
  if ((e = make_kmajor_map(&mb, b, eb, p.K, p.N, ldb * eb, BN / 2)) != cudaSuccess) return e;
  CUtensorMap mc;
  memset(&mc, 0, sizeof(mc));
  PeerMaps<GATHER> pm;
  memset(&pm, 0, sizeof(pm));
  if (TSTORE) {
    const int ob = (p.out_dtype == kF16 || p.out_dtype == kBF16) ? 2 : 4;
    if (!p.vec_ok) return cudaErrorInvalidValue;
    if ((e = make_out_map(&mc, p.out, ob, p.N, p.M, p.ldc * ob)) != cudaSuccess) return e;
    if constexpr (GATHER) {
      if (p.gather == kGatherTma)
        for (int q = 0; q < p.n_peers; ++q)
          if ((e = make_out_map(&pm.m[q], p.peer_out[q], ob, p.N, p.M, p.ldc * ob)) != cudaSuccess) return e;
    }
  }
  p.tiles_m = static_cast<int>((p.M + 255) / 256);
  p.tiles_n = static_cast<int>((p.N + BN - 1) / BN);
  const int tiles = p.tiles_m * p.tiles_n;
  int pairs = max_pairs[dev];
  if (max_ctas > 0 && max_ctas / 2 < pairs) pairs = max_ctas / 2 > 0 ? max_ctas / 2 : 1;
  if (tiles < pairs) pairs = tiles;
  cfg.gridDim = dim3(2 * pairs);
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, kernel, ma, mb, mc, pm, p);
  return e != cudaSuccess ? e : cudaGetLastError();
}

template <int KIND, int BT, int STAGES>
static cudaError_t launch_splitk(const void* a, int64_t lda, const void* b, int64_t ldb, GemmParams p,
                                 cudaStream_t stream) {
  using L = SplitSmem<BT, STAGES>;
  auto kernel = qgemm_splitk_kernel<KIND, BT, STAGES>;
  static bool configured[64] = {false};
  static int active[64][kSplitMax + 1] = {{0}};
  cudaError_t e = configure_once(kernel, L::kAlloc, configured);
  if (e != cudaSuccess) return e;
  const int dev = current_device();
  const int T = static_cast<int>((p.N + 127) / 128);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see griddep_wait
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = L::kAlloc;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // The largest split whose T clusters are all co-resident (one wave), at
  // most one CTA per k-block.
  int splits = 1;
  for (int s = kSplitMax; s >= 2; --s) {
    if (s > p.num_kb || T * s > device_sm_count()) continue;
    if (active[dev][s] == 0) {
      attr[0].val.clusterDim.x = s;
      cfg.gridDim = dim3(s * T);
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = -1;
      }
      active[dev][s] = n;
    }
    if (active[dev][s] >= T) {
      splits = s;
      break;
    }
  }
  const int eb = (KIND == kKindBF16 || KIND == kKindF16) ? 2 : 1;
  CUtensorMap mw, mx;
  if ((e = make_kmajor_map(&mw, b, eb, p.K, p.N, ldb * eb, 128)) != cudaSuccess) return e;
  if ((e = make_kmajor_map(&mx, a, eb, p.K, p.M, lda * eb, BT)) != cudaSuccess) return e;
  p.tiles_m = T;
  p.tiles_n = 1;
  attr[0].val.clusterDim.x = splits;
  cfg.gridDim = dim3(splits * T);
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, kernel, mw, mx, p);
  return e != cudaSuccess ? e : cudaGetLastError();
}

// Co-resident 2-CTA clusters of the pair kernel on the current device (the
// persistent grid size in pairs), or -1 when cluster launch is unavailable.
int pair_capacity() {
  using L = Smem<128, 128, 256, 7>;
  auto kernel = qgemm_pair_kernel<kKindI8, 256, 7, false>;
  static bool configured[64] = {false};
  static int cap[64] = {0};
  const int dev = current_device();
  if (dev >= 64) return -1;
  if (cap[dev] != 0) return cap[dev];
  if (configure_once(kernel, L::kAlloc, configured) != cudaSuccess) {
    cudaGetLastError();
    return cap[dev] = -1;
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * (device_sm_count() / 2));
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = L::kAlloc;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = -1;
  }
  return cap[dev] = n;
}

// Choose between 128x256 single-CTA tiles and 256x256 pair tiles by the
// modelled time of their persistent waves; pair tiles cost ~5% less per
// MAC (half the B operand per SM from shared memory and L2).
static int choose_config(int64_t M, int64_t N) {
  const int64_t tn = (N + 255) / 256;
  const int64_t t1 = (M + 127) / 128 * tn;
  const int64_t w1 = (t1 + device_sm_count() - 1) / device_sm_count();
  const int pairs = pair_capacity();
  if (N <= 128 && M <= 128) return 4;
  if (pairs <= 0 || M <= 128) return N <= 128 ? 4 : 3;
  const int64_t t2 = (M + 255) / 256 * tn;
  const int64_t w2 = (t2 + pairs - 1) / pairs;
  // one pair wave does twice a single wave's rows in the same time
  return static_cast<double>(w2) * 0.95 < static_cast<double>(w1) ? 5 : 3;
}

// Kernel selection: 0 auto; 1 single-CTA (auto N tile); 2 pair (auto N tile);
// 3 single BN=256; 4 single BN=128; 5 pair BN=256; 6 pair BN=192;
// 7 pair BN=256 with the TMA-store epilogue (needs 16-byte aligned output rows);
// 8 split-K swap-AB cluster kernel (M <= 32 only); 9 pair BN=192 with the
// TMA-store epilogue.
static int g_force_path = 0;
static int g_gather_store = 0;  // 0 = default, else kGatherSm / kGatherTma

template <int KIND>
static cudaError_t dispatch(int cfg, const void* a, int64_t lda, const void* b, int64_t ldb,
                           const GemmParams& p, int max_ctas, cudaStream_t stream) {
  switch (cfg) {
    case 3: return launch_single<KIND, 256, 4>(a, lda, b, ldb, p, max_ctas, stream);
    case 4: return launch_single<KIND, 128, 6>(a, lda, b, ldb, p, max_ctas, stream);
    // 7 stages: the ring covers the ~2k-cycle refill (TMA after the slot's
    // MMAs complete) at 512 tensor cycles per k-block; 6 left a bubble per wrap.
    case 5: return launch_pair<KIND, 256, 7, false>(a, lda, b, ldb, p, max_ctas, stream);
    case 6: return launch_pair<KIND, 192, 7, false>(a, lda, b, ldb, p, max_ctas, stream);
    // 6 stages + 32 KiB of output staging
    case 7: return launch_pair<KIND, 256, 6, true>(a, lda, b, ldb, p, max_ctas, stream);
    case 9: return launch_pair<KIND, 192, 6, true>(a, lda, b, ldb, p, max_ctas, stream);
    case 8:
      return p.M <= 16 ? launch_splitk<KIND, 16, 8>(a, lda, b, ldb, p, stream)
                       : launch_splitk<KIND, 32, 5>(a, lda, b, ldb, p, stream);
    default: return cudaErrorInvalidValue;
  }
}

// Gather mode: the pair TMA-store kernel with peer stores, 256x256 or
// 256x192 tiles by the same wave model as the automatic choice.
static cudaError_t run_gather(int kind, const void* a, int64_t lda, const void* b, int64_t ldb,
                              const GemmParams& p, cudaStream_t stream) {
  if (!p.vec_ok || p.N % 64 != 0 || p.n_peers < 0 || p.n_peers > kMaxGatherPeers || !p.done_count)
    return cudaErrorInvalidValue;
  GemmParams q = p;
  q.gather = g_gather_store == 0 ? kGatherDefault : g_gather_store;
  const int pairs = pair_capacity();
  if (pairs <= 0) return cudaErrorNotSupported;
  const int64_t tm2 = (p.M + 255) / 256;
  const int64_t w256 = (tm2 * ((p.N + 255) / 256) + pairs - 1) / pairs;
  const int64_t w192 = (tm2 * ((p.N + 191) / 192) + pairs - 1) / pairs;
  const bool narrow = static_cast<double>(w192) * 192.0 * 1.06 < static_cast<double>(w256) * 256.0;
  if (kind == kKindI8)
    return narrow ? launch_pair<kKindI8, 192, 6, true, true>(a, lda, b, ldb, q, 0, stream)
                  : launch_pair<kKindI8, 256, 6, true, true>(a, lda, b, ldb, q, 0, stream);
  if (kind == kKindE4M3)
    return narrow ? launch_pair<kKindE4M3, 192, 6, true, true>(a, lda, b, ldb, q, 0, stream)
                  : launch_pair<kKindE4M3, 256, 6, true, true>(a, lda, b, ldb, q, 0, stream);
  return cudaErrorInvalidValue;
}

cudaError_t run_qgemm(int kind, const void* a, int64_t lda, const void* b, int64_t ldb, GemmParams p,
                      int max_ctas, cudaStream_t stream) {
  if (p.M == 0 || p.N == 0) return cudaSuccess;
  p.status = status_word_ptr();
  const int eb = (kind == kKindBF16 || kind == kKindF16) ? 2 : 1;
  const int kb_elems = 128 / eb;
  p.num_kb = static_cast<int>((p.K + kb_elems - 1) / kb_elems);
  if (p.gather) return run_gather(kind, a, lda, b, ldb, p, stream);
  int cfg = g_force_path;
  const int64_t tm = (p.M + 127) / 128;
  const bool wide = p.N > 128 && tm * ((p.N + 255) / 256) >= device_sm_count() / 2;
  if (cfg == 8 && p.M > 32) cfg = 0;  // split-K covers decode sizes only
  if (cfg == 0 && p.M <= 32) cfg = 8;
  if (cfg == 0) {
    cfg = choose_config(p.M, p.N);
    // Staged TMA stores: whole 128-byte lines instead of 32 half-sector
    // stores per warp instruction; on the config-2 GEMM 107.5 us against
    // 129.0 us for the 7-stage st.global epilogue on the same box.
    if (cfg == 5 && p.vec_ok) {
      cfg = 7;
      // 256x192 pair tiles when the waves of the two tile widths favour
      // them: modelled time = waves x tile width, 192 weighted by 1.06 for
      // its larger operand stream per MAC.  Graph-replayed A/B on one B200:
      // 1024x3072x3072 15.4 -> 12.7 us, 2048x5120x5120 53.2 -> 42.7 us,
      // 8192x3072x3072 67.2 -> 61.3 us; the config-2 GEMM stays on 256
      // (102.4 against 104.5 us).
      const int pairs = pair_capacity();
      const int64_t tm2 = (p.M + 255) / 256;
      const int64_t w256 = (tm2 * ((p.N + 255) / 256) + pairs - 1) / pairs;
      const int64_t w192 = (tm2 * ((p.N + 191) / 192) + pairs - 1) / pairs;
      if (pairs > 0 && static_cast<double>(w192) * 192.0 * 1.06 < static_cast<double>(w256) * 256.0) cfg = 9;
    }
  }
  if (cfg == 2) cfg = 5;
  if (cfg == 1) cfg = wide ? 3 : 4;
  if (cfg == 7 && !p.vec_ok) cfg = 5;  // TMA stores need 16-byte aligned output rows
  if (cfg == 9 && !p.vec_ok) cfg = 6;
  cudaError_t e = kind == kKindI8     ? dispatch<kKindI8>(cfg, a, lda, b, ldb, p, max_ctas, stream)
                  : kind == kKindE4M3 ? dispatch<kKindE4M3>(cfg, a, lda, b, ldb, p, max_ctas, stream)
                  : kind == kKindF16  ? dispatch<kKindF16>(cfg, a, lda, b, ldb, p, max_ctas, stream)
                                      : dispatch<kKindBF16>(cfg, a, lda, b, ldb, p, max_ctas, stream);
  if (e == cudaErrorNotSupported && cfg >= 5 && g_force_path == 0) {
    cfg = wide ? 3 : 4;  // cluster launch unavailable: single-CTA tiles
    e = kind == kKindI8     ? dispatch<kKindI8>(cfg, a, lda, b, ldb, p, max_ctas, stream)
        : kind == kKindE4M3 ? dispatch<kKindE4M3>(cfg, a, lda, b, ldb, p, max_ctas, stream)
        : kind == kKindF16  ? dispatch<kKindF16>(cfg, a, lda, b, ldb, p, max_ctas, stream)
                            : dispatch<kKindBF16>(cfg, a, lda, b, ldb, p, max_ctas, stream);
  }
  return e;
}

void set_gemm_path(int path) { g_force_path = path; }

void set_gather_store(int mode) { g_gather_store = mode; }

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
