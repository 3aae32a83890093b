// Activation prologue for sm_100a: optional orthonormal block-Hadamard
// rotation, per-row absmax and round-to-nearest-even quantization to INT8
// (scale = absmax/127) or e4m3 (scale = absmax/448), one pass over HBM.
//
// Replaces the Kitchen ConvRot + quantize_int8_rowwise pair called at
// production/MOSS_RDNA2_INT8/backend.py:112-122 and the row quantizer
// _quant_rows of rdna2_ops/fp8_weight_gemm_v06.py:76-92 (ties to even here).
//
// Two kernels give bit-identical codes and scales:
//   act_quant_lane_kernel  INT8 ties-to-even codes of 16/32-bit rows with
//                          K % 64 == 0 (the production path): one lane per
//                          64-element slice, butterflies below 64 inside the
//                          lane, an exact FMA-corrected quantizer.
//   act_quant_kernel       every mode (e4m3, the reference's _quant_rows,
//                          fp8 inputs, ragged or unaligned rows), below.
//
// act_quant_kernel layout: a row is split into 256-element segments; lane l of a warp holds
// elements [seg*256 + 8l, seg*256 + 8l + 8) of each of its SPW segments in
// registers (one 16-byte load per segment for 16-bit inputs).  WPR warps share
// a row when K > 16 segments.  The butterfly stages run in the fixed order
// h = 1, 2, 4 (inside a lane), 8..128 (lane shuffles), 256.. (across the
// warp's segments), each pair (i, i+h) -> (a+b, a-b) in fp32, followed by one
// multiply by fp32(1/sqrt(block)) -- the same operation sequence as the CPU
// oracle, so the codes and scales are bit-identical.
#include "b2_common.cuh"
#include "b2_internal.h"

namespace b2 {

// Raw 16-byte (two for fp32) chunk of 8 consecutive elements of one lane.
struct Raw8 {
  uint4 a, b;
};

template <int DT>
__device__ __forceinline__ void load_raw(const void* x, int64_t off, bool vec, int valid, Raw8& r) {
  if constexpr (DT == kE4M3 || DT == kE5M2) {
    uint32_t lo = 0, hi = 0;
    const uint8_t* b = static_cast<const uint8_t*>(x) + off;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t v = j < valid ? b[j] : 0u;
      if (j < 4) lo |= v << (8 * j);
      else hi |= v << (8 * (j - 4));
    }
    r.a = make_uint4(lo, hi, 0u, 0u);
    return;
  }
  if (vec && valid == 8) {
    if constexpr (DT == kF32) {
      const uint4* p = reinterpret_cast<const uint4*>(static_cast<const float*>(x) + off);
      r.a = __ldg(p);
      r.b = __ldg(p + 1);
    } else {
      r.a = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + off));
    }
  } else {
    // Ragged tail, unaligned rows or dead rows: element loads, zero padding.
    uint32_t w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float f = j < valid ? load_as_float(x, DT, off + j) : 0.0f;
      if constexpr (DT == kF32) {
        w[j] = __float_as_uint(f);
      } else if constexpr (DT == kF16) {
        w[j] = __half_as_ushort(__float2half_rn(f));  // exact: f came from fp16
      } else {
        w[j] = __bfloat16_as_ushort(__float2bfloat16_rn(f));
      }
    }
    if constexpr (DT == kF32) {
      r.a = make_uint4(w[0], w[1], w[2], w[3]);
      r.b = make_uint4(w[4], w[5], w[6], w[7]);
    } else {
      r.a = make_uint4(w[0] | (w[1] << 16), w[2] | (w[3] << 16), w[4] | (w[5] << 16),
                       w[6] | (w[7] << 16));
    }
  }
}

template <int DT>
__device__ __forceinline__ void unpack_raw(const Raw8& r, float (&v)[8]) {
  if constexpr (DT == kE4M3 || DT == kE5M2) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      v[j] = fp8_to_float(static_cast<uint8_t>(((j < 4 ? r.a.x : r.a.y) >> (8 * (j & 3))) & 0xffu), DT);
  } else if constexpr (DT == kF32) {
    v[0] = __uint_as_float(r.a.x); v[1] = __uint_as_float(r.a.y);
    v[2] = __uint_as_float(r.a.z); v[3] = __uint_as_float(r.a.w);
    v[4] = __uint_as_float(r.b.x); v[5] = __uint_as_float(r.b.y);
    v[6] = __uint_as_float(r.b.z); v[7] = __uint_as_float(r.b.w);
  } else {
    const uint32_t w[4] = {r.a.x, r.a.y, r.a.z, r.a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (DT == kF16) {
        const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
        v[2 * i] = __low2float(h);
        v[2 * i + 1] = __high2float(h);
      } else {
        const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
        v[2 * i] = __low2float(h);
        v[2 * i + 1] = __high2float(h);
      }
    }
  }
}

// Exact quantizers: clamp(rint(RN(v/s))) for int8, e4m3_rn_sat(RN(v/s)).
// Fast path multiplies by r = RN(1/s): y = RN(v*r) lies within 2^-22
// relative of the exact quotient, as does RN(v/s), and rounding to the
// target grid is monotone, so whenever y is farther than a safety margin
// from a rounding boundary both give the same code.  Near a boundary (a few
// elements in 10^4) the correctly rounded IEEE quotient decides.
__device__ __forceinline__ uint32_t slow_int8(float v, float s) {
  int q = __float2int_rn(__fdiv_rn(v, s));
  q = q > 127 ? 127 : (q < -127 ? -127 : q);
  return static_cast<uint32_t>(q) & 0xffu;
}

// Returns a word whose low byte is the int8 code.
__device__ __forceinline__ uint32_t quant_int8(float v, float s, float r, bool fast) {
  const float y = __fmul_rn(v, r);               // |y| <= 127 * (1 + 2^-22)
  const float m = __fadd_rn(y, 12582912.0f);     // 1.5 * 2^23: rounds y to an integer (ties even)
  const float n = __fsub_rn(m, 12582912.0f);     // rint(y), exact
  if (fast && fabsf(__fsub_rn(n, y)) < 0.4998779296875f) {  // 0.5 - 2^-13 margin
    return __float_as_uint(m);                   // low byte = n mod 256, |n| <= 127
  }
  return slow_int8(v, s);
}

__device__ __forceinline__ uint32_t quant_e4m3(float v, float s, float r, bool fast) {
  if (fast) {
    const float y = __fmul_rn(v, r);
    const float d = __fmul_rn(fabsf(y), 9.5367431640625e-07f);  // 2^-20 relative margin
    const uint32_t lo = __nv_cvt_float_to_fp8(__fsub_rn(y, d), __NV_SATFINITE, __NV_E4M3);
    const uint32_t hi = __nv_cvt_float_to_fp8(__fadd_rn(y, d), __NV_SATFINITE, __NV_E4M3);
    if (lo == hi) return lo;
  }
  return static_cast<uint32_t>(__nv_cvt_float_to_fp8(__fdiv_rn(v, s), __NV_SATFINITE, __NV_E4M3));
}

// The reference's in-repo row quantizer _quant_rows
// (rdna2_ops/fp8_weight_gemm_v06.py:87-90): z = x / step, then
// floor(z + 0.5) or ceil(z - 0.5) in fp32 (half away from zero, including the
// fp32 rounding of z +- 0.5), clamped to [-127, 127].
__device__ __forceinline__ uint32_t quant_rows_ref(float v, float s) {
  const float z = __fdiv_rn(v, s);
  float q = z >= 0.0f ? floorf(__fadd_rn(z, 0.5f)) : ceilf(__fsub_rn(z, 0.5f));
  q = fminf(fmaxf(q, -127.0f), 127.0f);
  return static_cast<uint32_t>(static_cast<int>(q)) & 0xffu;
}

template <int QUANT>
__device__ __forceinline__ uint32_t pack4(const float* v, float s, float r, bool fast) {
  uint32_t c[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    c[i] = QUANT == 0 ? quant_int8(v[i], s, r, fast)
         : QUANT == 1 ? quant_e4m3(v[i], s, r, fast)
                      : quant_rows_ref(v[i], s);
  return __byte_perm(__byte_perm(c[0], c[1], 0x0040), __byte_perm(c[2], c[3], 0x0040), 0x5410);
}

// Persistent grid-stride kernel: a CTA of 4 warps handles 4/wpr rows per
// iteration (wpr warps per row, SPW 256-element segments per warp), and
// prefetches the next iteration's segments into registers before rotating
// and quantizing the current ones.
template <int DT, int SPW, int QUANT>
__global__ void __launch_bounds__(128)
    act_quant_kernel(const void* __restrict__ x, int64_t ldx, int M, int K, int wpr, int block,
                     float inv, uint8_t* __restrict__ q, int64_t ldq, float* __restrict__ scale,
                     int vec_in, int vec_out, int early) {
  __shared__ float s_max[2][4];
  if (early) griddep_launch_dependents();  // the GEMM may set up while the codes are written
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = 4 / wpr;
  const int g = warp / wpr, part = warp % wpr;
  const int64_t seg0 = static_cast<int64_t>(part) * SPW;
  const int64_t row_step = static_cast<int64_t>(gridDim.x) * groups;

  auto issue = [&](int64_t row, Raw8 (&raw)[SPW]) {
    const bool live = row < M;
#pragma unroll
    for (int s = 0; s < SPW; ++s) {
      const int64_t k0 = (seg0 + s) * 256 + lane * 8;
      const int64_t rem = static_cast<int64_t>(K) - k0;
      const int valid = live ? static_cast<int>(rem < 0 ? 0 : (rem > 8 ? 8 : rem)) : 0;
      load_raw<DT>(x, live ? row * ldx + k0 : 0, vec_in != 0, valid, raw[s]);
    }
  };

  Raw8 raw[SPW];
  int64_t base = static_cast<int64_t>(blockIdx.x) * groups;
  issue(base + g, raw);
  int parity = 0;
  for (; base < M; base += row_step) {
    const int64_t row = base + g;
    const bool live = row < M;
    float v[SPW][8];
#pragma unroll
    for (int s = 0; s < SPW; ++s) unpack_raw<DT>(raw[s], v[s]);
    if (base + row_step < M) issue(base + row_step + g, raw);  // next rows in flight

    if (block > 1) {
#pragma unroll
      for (int h = 1; h < 8; h <<= 1) {
        if (block > h) {
#pragma unroll
          for (int s = 0; s < SPW; ++s)
#pragma unroll
            for (int i = 0; i < 8; ++i)
              if (!(i & h)) {
                const float a = v[s][i], b = v[s][i + h];
                v[s][i] = __fadd_rn(a, b);
                v[s][i + h] = __fsub_rn(a, b);
              }
        }
      }
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        if (block > 8 * d) {
          // lower lane: v + o; upper lane: o - v.  fma(+-1, v, o) rounds once,
          // exactly like the add/sub it replaces.
          const float sgn = (lane & d) ? -1.0f : 1.0f;
#pragma unroll
          for (int s = 0; s < SPW; ++s)
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float o = __shfl_xor_sync(0xffffffffu, v[s][i], d);
              v[s][i] = __fmaf_rn(sgn, v[s][i], o);
            }
        }
      }
#pragma unroll
      for (int ds = 1; ds < SPW; ds <<= 1) {
        if (block > 256 * ds) {
#pragma unroll
          for (int s = 0; s < SPW; ++s)
            if (!(s & ds) && s + ds < SPW) {
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const float a = v[s][i], b = v[s + ds][i];
                v[s][i] = __fadd_rn(a, b);
                v[s + ds][i] = __fsub_rn(a, b);
              }
            }
        }
      }
#pragma unroll
      for (int s = 0; s < SPW; ++s)
#pragma unroll
        for (int i = 0; i < 8; ++i) v[s][i] = __fmul_rn(v[s][i], inv);
    }

    float amax = 0.0f;
#pragma unroll
    for (int s = 0; s < SPW; ++s)
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[s][i]));
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, d));
    if (wpr > 1) {
      if (lane == 0) s_max[parity][warp] = amax;
      __syncthreads();
      for (int w = 0; w < wpr; ++w) amax = fmaxf(amax, s_max[parity][g * wpr + w]);
      parity ^= 1;
    }
    float sc = __fdiv_rn(amax, QUANT == 1 ? 448.0f : 127.0f);
    if constexpr (QUANT == 2) {
      sc = fmaxf(sc, 1.0e-20f);                    // step floor of _quant_rows
    } else {
      if (!(sc > 0.0f)) sc = 1.0f;
    }
    if (!live) continue;
    const float rcp = __frcp_rn(sc);
    const bool fast = sc > 1e-30f && sc < 1e30f;

#pragma unroll
    for (int s = 0; s < SPW; ++s) {
      const int64_t k0 = (seg0 + s) * 256 + lane * 8;
      if (k0 >= K) continue;
      uint8_t* dst = q + row * ldq + k0;
      const uint32_t lo = pack4<QUANT>(&v[s][0], sc, rcp, fast);
      const uint32_t hi = pack4<QUANT>(&v[s][4], sc, rcp, fast);
      if (vec_out && k0 + 8 <= K) {
        *reinterpret_cast<uint2*>(dst) = make_uint2(lo, hi);
      } else {
        for (int i = 0; i < 8 && k0 + i < K; ++i)
          dst[i] = static_cast<uint8_t>((i < 4 ? lo >> (8 * i) : hi >> (8 * (i - 4))) & 0xffu);
      }
    }
    if (part == 0 && lane == 0) scale[row] = sc;
  }
}

// ------------------------------------------------------- lane-block kernel
// INT8 (ties-to-even) prologue with one lane per E-element slice of a row:
// every butterfly stage below E runs inside the lane (one add or subtract
// per element, no shuffles), stages E..block/2 exchange with the lane
// (h / E) away, and the per-row absmax meets in shared memory.  Rows of
// TPR = K / E lanes are packed R to a CTA.
//
// Quantization is exact without a slow path: with r = RN(1/s) (correctly
// rounded reciprocal), y = RN(v*r) is a faithful approximation of v/s, the
// residual e = v - s*y is exact in one fma, and RN(y + e*r) is the correctly
// rounded quotient RN(v/s) (Markstein's theorem, IBM J. Res. Dev. 34(1),
// 1990; Muller et al., Handbook of Floating-Point Arithmetic, 2nd ed.,
// section 5.1).  Its conditions (no overflow, no underflow of the residual
// for quotients that can reach 1/2) hold for s in [2^-60, 2^60]; rows
// outside that range are rescaled by an exact power of two (2^64 or 2^-64,
// applied to v and s alike), which leaves every quotient that can round
// away from zero unchanged.  Rows with a non-finite scale use the IEEE
// division per element.  E = 64 elements per lane; a CTA holds whole rows
// (about 128 threads, at most kLaneThreads), several CTAs per SM.
constexpr int kLaneE = 64;
constexpr int kLaneThreads = 384;
constexpr int kLaneFull = 0;
constexpr int kLaneAmax = 1;
constexpr int kLaneCodes = 2;
constexpr int kLaneFused = 3;

// End of a sharded-mode launch, run by every thread: orders this thread's
// peer stores, counts the CTA, and the last CTA releases the epoch into slot
// `rank` of every rank's flag array and rearms the counter.
__device__ __forceinline__ void shard_signal_to(int world, uint32_t* const* flag_slot, uint32_t* done_count,
                                                uint32_t epoch) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(done_count, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      for (int r = 0; r < world; ++r) st_release_sys(flag_slot[r], epoch);
      *done_count = 0u;
    }
  }
}

__device__ __forceinline__ void shard_signal(const ShardArgs& sh) {
  shard_signal_to(sh.world, sh.flag_slot, sh.done_count, sh.epoch);
}

// Fused mode, between the two passes: signal the absmax phase like
// shard_signal, then wait (bounded, one thread per CTA) until every rank's
// absmax slots for this epoch have arrived.  Needs every CTA of the grid
// resident (cooperative launch): a waiting CTA never blocks one that has
// yet to signal.  CTA-uniform result; false after the wait limit (status
// 0x100 | kSiteGather).
__device__ __forceinline__ bool shard_barrier(const ShardArgs& sh) {
  __shared__ int s_ok;
  shard_signal(sh);
  if (threadIdx.x == 0) {
    int ok = 1;
    const uint64_t start = globaltimer();
    for (int r = 0; r < sh.world && ok; ++r) {
      for (uint32_t i = 0;; ++i) {
        if (static_cast<int32_t>(ld_acquire_sys(sh.own_flags + r) - sh.epoch) >= 0) break;
        if ((i & 255u) == 255u && globaltimer() - start > kWaitLimitNs) {
          if (sh.status != nullptr) atomicCAS(sh.status, 0, 0x100 | kSiteGather);
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// A sharded launch whose slice is empty (this rank holds none of the next
// layer's input columns): kLaneAmax writes 0 into its slots (the absmax of
// nothing; 0 never raises a maximum of absolute values), kLaneCodes only
// computes the row scales from the exchanged maxima.
template <bool FP8>
__global__ void shard_empty_kernel(int mode, int M, float* __restrict__ scale, const ShardArgs sh) {
  for (int row = blockIdx.x * blockDim.x + threadIdx.x; row < M; row += gridDim.x * blockDim.x) {
    if (mode == kLaneAmax) {
      for (int r = 0; r < sh.world; ++r) sh.xchg[r][static_cast<int64_t>(sh.rank) * M + row] = 0.0f;
    } else {
      float amax = 0.0f;
      for (int r = 0; r < sh.world; ++r) amax = fmaxf(amax, sh.xlocal[static_cast<int64_t>(r) * M + row]);
      float sc = __fdiv_rn(amax, FP8 ? 448.0f : 127.0f);
      if (!(sc > 0.0f)) sc = 1.0f;
      scale[row] = sc;
    }
  }
  shard_signal(sh);
}

template <int DT, int E>
__device__ __forceinline__ void load_slice(const void* x, int64_t off, bool live, float (&v)[E]) {
  if (!live) {
#pragma unroll
    for (int i = 0; i < E; ++i) v[i] = 0.0f;
    return;
  }
  if constexpr (DT == kF32) {
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const float*>(x) + off);
#pragma unroll
    for (int j = 0; j < E / 4; ++j) {
      const uint4 w = __ldg(p + j);
      v[4 * j] = __uint_as_float(w.x);
      v[4 * j + 1] = __uint_as_float(w.y);
      v[4 * j + 2] = __uint_as_float(w.z);
      v[4 * j + 3] = __uint_as_float(w.w);
    }
  } else {
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + off);
    uint4 w[E / 8];
#pragma unroll
    for (int j = 0; j < E / 8; ++j) w[j] = __ldg(p + j);
#pragma unroll
    for (int j = 0; j < E / 8; ++j) {
      Raw8 r;
      r.a = w[j];
      float f[8];
      unpack_raw<DT>(r, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[8 * j + i] = f[i];
    }
  }
}

__device__ __forceinline__ uint32_t code_markstein(float v, float s, float r) {
  const float y = __fmul_rn(v, r);
  const float e = __fmaf_rn(-s, y, v);       // exact residual
  const float z = __fmaf_rn(e, r, y);        // RN(v / s)
  return __float_as_uint(__fadd_rn(z, 12582912.0f));  // low byte = rint(z), |z| <= 127
}

// Modes of the lane kernel.  kLaneFull: codes and scales of whole rows.
// The two sharded modes serve a column-parallel layer whose next layer reads
// the whole row: each rank holds a column slice of the row (whole rotation
// blocks), kLaneAmax writes the slice's absmax of the rotated values into
// slot `rank` of every rank's exchange buffer [world][M]; kLaneCodes takes
// the row's absmax as the maximum over the world slots (exactly the whole
// row's absmax: max is exact), and writes the slice's codes into the same
// columns of every rank's code buffer and the row scale locally.  Codes and
// scales are bit-identical to kLaneFull on the whole row.  Both sharded
// modes end with the gather signal: a system-scope fence, a CTA count, and
// the last CTA releasing `epoch` into slot `rank` of every rank's flags.

template <int DT, bool FP8 = false, int E = kLaneE, int MODE = kLaneFull>
__global__ void __launch_bounds__(kLaneThreads, 1)
    act_quant_lane_kernel(const void* __restrict__ x, int64_t ldx, int M, int K, int tpr, int rows_per_cta,
                          int block, float inv, uint8_t* __restrict__ q, int64_t ldq, float* __restrict__ scale,
                          int early, const ShardArgs sh) {
  __shared__ uint32_t s_max[3][kLaneThreads];
  // kLaneCodes: the CTA's codes are staged in shared memory (two buffers of
  // rows_per_cta x K bytes) and each row leaves as one bulk store per rank,
  // issued by the row's first lane after the next CTA barrier, so that the
  // stores to the peers stream while the next rows are rotated.
  extern __shared__ __align__(128) uint8_t s_stage[];
  if (early) griddep_launch_dependents();  // the GEMM may set up while the codes are written
  const int tid = threadIdx.x;
  const int r_local = tid / tpr;
  const int part = tid - r_local * tpr;
  const bool active = r_local < rows_per_cta;
  const int lane = tid & 31;
  const int64_t row_step = static_cast<int64_t>(gridDim.x) * rows_per_cta;
  int64_t staged_row = -1;  // kLaneCodes, first lane of a row: the row staged in the previous iteration
  auto send_row = [&](int buf) {
    const uint32_t src = smem_u32(s_stage) + static_cast<uint32_t>((buf * rows_per_cta + r_local) * K);
    for (int r = 0; r < sh.world; ++r) bulk_store(sh.qout[r] + staged_row * ldq, src, static_cast<uint32_t>(K));
    bulk_commit_group();
  };
  for (int i = tid; i < 3 * kLaneThreads; i += blockDim.x) (&s_max[0][0])[i] = 0u;
  // 16-bit rows with E = 64: the next row group's slice (32 registers) is in
  // flight while the current one is rotated and quantized.
  constexpr bool kPrefetch = DT != kF32 && E == 64;
  uint4 raw[kPrefetch ? E / 8 : 1];
  auto issue = [&](int64_t b) {
    const int64_t rw = b + r_local;
    const bool lv = active && rw < M;
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) +
                                                    (lv ? rw * ldx + static_cast<int64_t>(part) * E : 0));
#pragma unroll
    for (int j = 0; j < (kPrefetch ? E / 8 : 1); ++j) raw[j] = lv ? __ldg(p + j) : make_uint4(0u, 0u, 0u, 0u);
  };
  if constexpr (kPrefetch) issue(static_cast<int64_t>(blockIdx.x) * rows_per_cta);
  __syncthreads();
  int it = 0;
  constexpr bool kFused = MODE == kLaneFused;
  bool fused_ok = true;  // CTA-uniform: the barrier between the passes completed
  for (int pass = 0; pass < (kFused ? 2 : 1); ++pass) {
  // amax pass: the slice's row maxima to every rank; codes pass: codes with
  // the row's global scale, staged and sent by bulk stores
  const bool amax_pass = MODE == kLaneAmax || (kFused && pass == 0);
  const bool codes_pass = MODE == kLaneCodes || (kFused && pass == 1);
  if (kFused && pass == 1) {
    if (!shard_barrier(sh)) {
      fused_ok = false;  // no codes: release nothing, the peers' waits give up too
      break;
    }
    if constexpr (kPrefetch) issue(static_cast<int64_t>(blockIdx.x) * rows_per_cta);
  }
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * rows_per_cta; base < M; base += row_step, ++it) {
    const int64_t row = base + r_local;
    const bool live = active && row < M;
    // The slice lives in element pairs: every butterfly stage from h = 2
    // up, the 1/sqrt(B) scaling and the quantizer run on Blackwell's packed
    // fp32 instructions (two lanes per instruction, each lane rounded exactly
    // like the scalar operation it replaces).  No packed multiply feeds a
    // packed add here: such a pair was measured to come out fused (one
    // rounding) elsewhere, which the exact codes could not tolerate.
    float2 w[E / 2];
    if constexpr (kPrefetch) {
#pragma unroll
      for (int j = 0; j < E / 8; ++j) {
        Raw8 r8;
        r8.a = raw[j];
        float f[8];
        unpack_raw<DT>(r8, f);
#pragma unroll
        for (int i = 0; i < 4; ++i) w[4 * j + i] = make_float2(f[2 * i], f[2 * i + 1]);
      }
      if (base + row_step < M) issue(base + row_step);
    } else {
      float v[E];
      load_slice<DT, E>(x, live ? row * ldx + static_cast<int64_t>(part) * E : 0, live, v);
#pragma unroll
      for (int i = 0; i < E / 2; ++i) w[i] = make_float2(v[2 * i], v[2 * i + 1]);
    }

    if (block > 1) {
      // h = 1: the two elements of a pair
#pragma unroll
      for (int i = 0; i < E / 2; ++i) {
        const float a = w[i].x, b = w[i].y;
        w[i] = make_float2(__fadd_rn(a, b), __fsub_rn(a, b));
      }
      // h = 2H for H = 1, 2, ...: pair i with pair i + H; a - b as
      // fma(b, -1, a), one rounding of the exact difference.
      const float2 neg1 = make_float2(-1.0f, -1.0f);
#pragma unroll
      for (int H = 1; 2 * H < E; H <<= 1) {
        if (block > 2 * H) {
#pragma unroll
          for (int i = 0; i < E / 2; ++i)
            if (!(i & H)) {
              const float2 a = w[i], b = w[i + H];
              w[i] = __fadd2_rn(a, b);
              w[i + H] = __ffma2_rn(b, neg1, a);
            }
        }
      }
      // stages h = E .. block/2: partner lane (h / E) away (same warp: the
      // lanes of one block are consecutive and aligned); lower lane a + b,
      // upper lane a - b with a the lower lane's value.
      for (int d = 1; d * E < block; d <<= 1) {
        const float sg = (lane & d) ? -1.0f : 1.0f;
        const float2 sg2 = make_float2(sg, sg);
#pragma unroll
        for (int i = 0; i < E / 2; ++i) {
          const float2 o = make_float2(__shfl_xor_sync(0xffffffffu, w[i].x, d),
                                       __shfl_xor_sync(0xffffffffu, w[i].y, d));
          w[i] = __ffma2_rn(w[i], sg2, o);
        }
      }
      const float2 inv2 = make_float2(inv, inv);
#pragma unroll
      for (int i = 0; i < E / 2; ++i) w[i] = __fmul2_rn(w[i], inv2);
    }

    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < E / 2; ++i) amax = fmaxf(fmaxf(amax, fabsf(w[i].x)), fabsf(w[i].y));
    const int sb = it % 3;
    if (live) atomicMax(&s_max[sb][r_local], __float_as_uint(amax));
    for (int i = tid; i < rows_per_cta; i += blockDim.x) s_max[(it + 1) % 3][i] = 0u;  // next iteration's
    if (codes_pass) {
      if (part == 0 && active) bulk_wait_read<0>();  // this iteration's buffer is free again
    }
    __syncthreads();
    if (codes_pass) {
      if (part == 0 && active) {
        if (staged_row >= 0) send_row((it + 1) & 1);
        staged_row = live ? row : -1;
      }
    }
    if (!live) continue;
    amax = __uint_as_float(s_max[sb][r_local]);
    if (amax_pass) {
      if (part == 0)
        for (int r = 0; r < sh.world; ++r) sh.xchg[r][static_cast<int64_t>(sh.rank) * M + row] = amax;
      continue;
    }
    if (codes_pass) {
      amax = 0.0f;
      for (int r = 0; r < sh.world; ++r) amax = fmaxf(amax, sh.xlocal[static_cast<int64_t>(r) * M + row]);
    }
    float sc = __fdiv_rn(amax, FP8 ? 448.0f : 127.0f);
    if (!(sc > 0.0f)) sc = 1.0f;

    uint8_t* dst = q + row * ldq + static_cast<int64_t>(part) * E;
    uint8_t* stage = s_stage + ((it & 1) * rows_per_cta + r_local) * K + part * E;
    auto put = [&](int j, const uint4& v) {
      if (codes_pass) {
        *reinterpret_cast<uint4*>(stage + 16 * j) = v;
      } else {
        *reinterpret_cast<uint4*>(dst + 16 * j) = v;
      }
    };
    // Normal, finite scales: |RN(v/s)| <= 127 with no clamp needed, since
    // s = RN(absmax/127) carries a relative error below 2^-24.  Subnormal
    // scales lose that precision (quotients can exceed 127.5) and take the
    // clamped IEEE division, like non-finite ones.
    const bool exact_path = sc >= 1.1754943508222875e-38f && sc <= 3.4028234663852886e38f;
    if (exact_path) {
      float s2 = sc;
      if (sc < 8.673617379884035e-19f) {         // 2^-60
        s2 = __fmul_rn(sc, 1.8446744073709552e19f);  // x 2^64, exact
        const float2 k2 = make_float2(1.8446744073709552e19f, 1.8446744073709552e19f);
#pragma unroll
        for (int i = 0; i < E / 2; ++i) w[i] = __fmul2_rn(w[i], k2);
      } else if (sc > 1.152921504606847e18f) {   // 2^60
        s2 = __fmul_rn(sc, 5.421010862427522e-20f);  // x 2^-64, exact for s
        const float2 k2 = make_float2(5.421010862427522e-20f, 5.421010862427522e-20f);
#pragma unroll
        for (int i = 0; i < E / 2; ++i) w[i] = __fmul2_rn(w[i], k2);
      }
      const float r = __frcp_rn(s2);
      const float2 r2 = make_float2(r, r), ns2 = make_float2(-s2, -s2);
      const float2 magic = make_float2(12582912.0f, 12582912.0f);
      // the exact quotient of the pair i (Markstein, as code_markstein):
      // y = v*r, e = v - s*y exactly, RN(v/s) = y + e*r
      auto quotient = [&](int i) {
        const float2 y = __fmul2_rn(w[i], r2);
        const float2 e = __ffma2_rn(ns2, y, w[i]);
        return __ffma2_rn(e, r2, y);
      };
      // int8: + 1.5*2^23 leaves the ties-to-even integer in the low byte
      auto codes = [&](int i, uint32_t& lo, uint32_t& hi) {
        const float2 m = __fadd2_rn(quotient(i), magic);
        lo = __float_as_uint(m.x);
        hi = __float_as_uint(m.y);
      };
      // e4m3: one round-to-nearest-even, saturating conversion of the pair
      // (e4m3_rn_sat(RN(v/s)), the oracle's b2o_f32_to_e4m3).  The quotient
      // takes v's sign: RN(v/s) has it for every v (s > 0), but the FMA
      // correction turns a -0 input into +0, and e4m3 keeps the sign of zero.
      auto codes_e4m3 = [&](int i) {
        float2 z = quotient(i);
        z.x = copysignf(z.x, w[i].x);
        z.y = copysignf(z.y, w[i].y);
        return static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(z, __NV_SATFINITE, __NV_E4M3));
      };
#pragma unroll
      for (int j = 0; j < E / 16; ++j) {
        uint32_t o[4];
#pragma unroll
        for (int t2 = 0; t2 < 4; ++t2) {
          if constexpr (FP8) {
            o[t2] = codes_e4m3(8 * j + 2 * t2) | (codes_e4m3(8 * j + 2 * t2 + 1) << 16);
          } else {
            uint32_t c0, c1, c2, c3;
            codes(8 * j + 2 * t2, c0, c1);
            codes(8 * j + 2 * t2 + 1, c2, c3);
            o[t2] = __byte_perm(__byte_perm(c0, c1, 0x0040), __byte_perm(c2, c3, 0x0040), 0x5410);
          }
        }
        put(j, make_uint4(o[0], o[1], o[2], o[3]));
      }
    } else {
#pragma unroll
      for (int j = 0; j < E / 16; ++j) {
        uint32_t o[4];
#pragma unroll
        for (int t2 = 0; t2 < 4; ++t2) {
          const float2 p0 = w[8 * j + 2 * t2], p1 = w[8 * j + 2 * t2 + 1];
          if constexpr (FP8) {
            o[t2] = quant_e4m3(p0.x, sc, 0.0f, false) | (quant_e4m3(p0.y, sc, 0.0f, false) << 8) |
                    (quant_e4m3(p1.x, sc, 0.0f, false) << 16) | (quant_e4m3(p1.y, sc, 0.0f, false) << 24);
          } else {
            o[t2] = __byte_perm(__byte_perm(slow_int8(p0.x, sc), slow_int8(p0.y, sc), 0x0040),
                                __byte_perm(slow_int8(p1.x, sc), slow_int8(p1.y, sc), 0x0040), 0x5410);
          }
        }
        put(j, make_uint4(o[0], o[1], o[2], o[3]));
      }
    }
    if (part == 0) scale[row] = sc;
    if (codes_pass) fence_proxy_async_smem();  // staged codes visible to the bulk stores
  }
  }
  if constexpr (MODE == kLaneCodes || kFused) {
    __syncthreads();
    if (part == 0 && active) {
      if (staged_row >= 0) send_row((it + 1) & 1);
      bulk_wait_all();               // every row at every rank
      fence_proxy_async_global();
    }
  }
  if constexpr (kFused) {
    if (fused_ok) shard_signal_to(sh.world, sh.flag_slot2, sh.done_count2, sh.epoch2);
  } else if constexpr (MODE != kLaneFull) {
    shard_signal(sh);
  }
}

// 0 automatic (the lane-block kernel where it applies, else the warp-shuffle
// kernel), 1 warp-shuffle kernel, 2 lane-block kernel (a verification and
// tuning knob).
static int g_prologue_path = 0;
void set_prologue_path(int path) { g_prologue_path = path; }

// Small CTAs (about 128 threads: whole rows of TPR lanes), several per SM,
// so that one CTA's loads overlap another's arithmetic across the per-row
// barrier.
template <int DT, bool FP8, int MODE = kLaneFull>
static cudaError_t launch_lane(int64_t M, cudaStream_t st, const void* x, int64_t ldx, int K, int block,
                               float inv, uint8_t* q, int64_t ldq, float* scale, int early,
                               const ShardArgs& sh = ShardArgs{}) {
  auto kernel = act_quant_lane_kernel<DT, FP8, kLaneE, MODE>;
  const int tpr = K / kLaneE;
  int rows = 128 / tpr;
  if (rows < 1) rows = 1;
  const int threads = (rows * tpr + 31) / 32 * 32;
  // kLaneCodes stages two buffers of rows x K code bytes (at most 48 KiB)
  const size_t dyn = (MODE == kLaneCodes || MODE == kLaneFused) ? static_cast<size_t>(2 * rows * K) : 0;
  if (MODE == kLaneCodes || MODE == kLaneFused) {
    static bool configured[64] = {false};
    int d = 0;
    cudaGetDevice(&d);
    if (d < 64 && !configured[d]) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * 384 * kLaneE);
      if (e != cudaSuccess) return e;
      configured[d] = true;
    }
  }
  static int per_sm[64][8] = {{0}};
  int dev = 0;
  cudaGetDevice(&dev);
  const int slot = threads / 32 - 1;  // 1..12 warps -> slot 0..11; cache the common ones
  int n = 0;
  if (dev < 64 && slot < 8 && per_sm[dev][slot] > 0) {
    n = per_sm[dev][slot];
  } else {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, dyn) != cudaSuccess || n <= 0) n = 1;
    if (dev < 64 && slot < 8) per_sm[dev][slot] = n;
  }
  const int64_t need = (M + rows - 1) / rows;
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * n;
  const unsigned grid = static_cast<unsigned>(need < cap ? need : cap);
  if constexpr (MODE == kLaneFused) {
    // every CTA resident at once: the CTAs wait for one another (through
    // the other ranks) between the passes
    int m32 = static_cast<int>(M);
    void* args[] = {(void*)&x, (void*)&ldx, (void*)&m32, (void*)&K, (void*)&tpr, (void*)&rows, (void*)&block,
                    (void*)&inv, (void*)&q, (void*)&ldq, (void*)&scale, (void*)&early, (void*)&sh};
    cudaError_t e = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(kernel), dim3(grid), dim3(threads),
                                                args, dyn, st);
    return e != cudaSuccess ? e : cudaGetLastError();
  }
  kernel<<<grid, threads, dyn, st>>>(x, ldx, static_cast<int>(M), K, tpr, rows, block, inv, q, ldq, scale, early,
                                     sh);
  return cudaGetLastError();
}

// The lane-block kernel applies to INT8 ties-to-even codes of 16/32-bit
// inputs whose rows split into whole 64-element slices (at most
// kLaneThreads), with 16-byte aligned input and code rows and rotation
// blocks of at most 32 lanes.
static bool lane_ok(int x_dtype, int quant, int64_t K, int block, bool vin16, bool vout16) {
  if (quant > 1 || !(x_dtype == kF16 || x_dtype == kBF16 || x_dtype == kF32)) return false;
  if (!vin16 || !vout16 || K % kLaneE != 0 || K / kLaneE > kLaneThreads) return false;
  return block <= 1 || block <= 32 * kLaneE;
}

template <int DT, int SPW, int QUANT>
static cudaError_t launch_one(int early, int64_t M, cudaStream_t st, const void* x, int64_t ldx, int K, int wpr,
                              int block, float inv, uint8_t* q, int64_t ldq, float* scale, int vin,
                              int vout) {
  auto kernel = act_quant_kernel<DT, SPW, QUANT>;
  static int per_sm[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && per_sm[dev] == 0) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, 128, 0) != cudaSuccess || n <= 0) n = 4;
    per_sm[dev] = n;
  }
  const int groups = 4 / wpr;
  const int64_t need = (M + groups - 1) / groups;
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * (dev < 64 ? per_sm[dev] : 4);
  const unsigned grid = static_cast<unsigned>(need < cap ? need : cap);
  kernel<<<grid, 128, 0, st>>>(x, ldx, static_cast<int>(M), K, wpr, block, inv, q, ldq, scale, vin, vout,
                               early);
  return cudaGetLastError();
}

template <int DT, int QUANT>
static cudaError_t launch_spw(int early, int spw, int64_t M, cudaStream_t st, const void* x, int64_t ldx, int K,
                             int wpr, int block, float inv, uint8_t* q, int64_t ldq, float* scale,
                             int vin, int vout) {
#define B2_SPW_CASE(S) \
  case S:              \
    return launch_one<DT, S, QUANT>(early, M, st, x, ldx, K, wpr, block, inv, q, ldq, scale, vin, vout);
  switch (spw) {
    B2_SPW_CASE(1) B2_SPW_CASE(2) B2_SPW_CASE(3) B2_SPW_CASE(4) B2_SPW_CASE(5) B2_SPW_CASE(6)
    B2_SPW_CASE(7) B2_SPW_CASE(8) B2_SPW_CASE(10) B2_SPW_CASE(12) B2_SPW_CASE(16)
    default: return cudaErrorInvalidValue;
  }
#undef B2_SPW_CASE
}

// Pick warps-per-row and segments-per-warp: the fewest segments per lane
// (registers, hence occupancy) that cover the row with up to 4 warps, warp
// ranges aligned to the rotation block.
static bool choose_layout(int64_t K, int block, int* wpr, int* spw) {
  static const int kSpw[] = {1, 2, 3, 4, 5, 6, 7, 8, 10, 12, 16};
  for (int s : kSpw) {
    for (int w : {1, 2, 4}) {
      if (static_cast<int64_t>(w) * s * 256 < K) continue;
      if (block > 1 && block > s * 256) continue;
      if (block > 1 && w > 1 && (s * 256) % block != 0) continue;
      *wpr = w;
      *spw = s;
      return true;
    }
  }
  return false;
}

cudaError_t run_act_quant(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int block,
                          int quant, void* q, int64_t ldq, float* scale, cudaStream_t stream,
                          bool early_dependents) {
  if (M == 0) return cudaSuccess;
  const int early = early_dependents ? 1 : 0;
  const int eb = x_dtype == kF32 ? 4 : (x_dtype == kE4M3 || x_dtype == kE5M2) ? 1 : 2;
  const float inv_b = block > 1 ? static_cast<float>(1.0 / sqrt(static_cast<double>(block))) : 1.0f;
  {
    const bool vin16 = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && ((ldx * eb) % 16 == 0);
    const bool vout16 = (reinterpret_cast<uintptr_t>(q) % 16 == 0) && (ldq % 16 == 0);
    if (g_prologue_path != 1 && lane_ok(x_dtype, quant, K, block, vin16, vout16)) {
      uint8_t* qb = static_cast<uint8_t*>(q);
      const int k = static_cast<int>(K);
      if (quant == 1) {
        switch (x_dtype) {
          case kF32: return launch_lane<kF32, true>(M, stream, x, ldx, k, block, inv_b, qb, ldq, scale, early);
          case kF16: return launch_lane<kF16, true>(M, stream, x, ldx, k, block, inv_b, qb, ldq, scale, early);
          default: return launch_lane<kBF16, true>(M, stream, x, ldx, k, block, inv_b, qb, ldq, scale, early);
        }
      }
      switch (x_dtype) {
        case kF32: return launch_lane<kF32, false>(M, stream, x, ldx, k, block, inv_b, qb, ldq, scale, early);
        case kF16: return launch_lane<kF16, false>(M, stream, x, ldx, k, block, inv_b, qb, ldq, scale, early);
        default: return launch_lane<kBF16, false>(M, stream, x, ldx, k, block, inv_b, qb, ldq, scale, early);
      }
    }
  }
  int wpr = 1, spw = 1;
  if (!choose_layout(K, block, &wpr, &spw)) return cudaErrorInvalidValue;
  const int vin = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && ((ldx * eb) % 16 == 0);
  const int vout = (reinterpret_cast<uintptr_t>(q) % 8 == 0) && (ldq % 8 == 0);
  const float inv = block > 1 ? static_cast<float>(1.0 / sqrt(static_cast<double>(block))) : 1.0f;
  uint8_t* qb = static_cast<uint8_t*>(q);
  const int k = static_cast<int>(K);
#define B2_AQ(DT, Q) \
  return launch_spw<DT, Q>(early, spw, M, stream, x, ldx, k, wpr, block, inv, qb, ldq, scale, vin, vout)
#define B2_AQ_DT(Q)                 \
  switch (x_dtype) {                \
    case kF32: B2_AQ(kF32, Q);      \
    case kF16: B2_AQ(kF16, Q);      \
    case kBF16: B2_AQ(kBF16, Q);    \
    case kE4M3: B2_AQ(kE4M3, Q);    \
    case kE5M2: B2_AQ(kE5M2, Q);    \
    default: return cudaErrorInvalidValue; \
  }
  if (quant == 0) { B2_AQ_DT(0) }
  if (quant == 1) { B2_AQ_DT(1) }
  B2_AQ_DT(2)
#undef B2_AQ_DT
#undef B2_AQ
}

cudaError_t run_shard_quant(int mode, const void* y, int y_dtype, int64_t M, int64_t Ns, int64_t ldy, int block,
                            int quant, int64_t ldq, float* scale, const ShardArgs& sh, cudaStream_t stream) {
  if (M <= 0) return cudaSuccess;
  if (mode != kLaneAmax && mode != kLaneCodes && mode != kLaneFused) return cudaErrorInvalidValue;
  if (mode == kLaneFused && Ns == 0) return cudaErrorInvalidValue;
  if (Ns == 0) {
    const int64_t blocks = (M + 255) / 256;
    const unsigned grid = static_cast<unsigned>(blocks < 1024 ? blocks : 1024);
    if (quant == 1)
      shard_empty_kernel<true><<<grid, 256, 0, stream>>>(mode, static_cast<int>(M), scale, sh);
    else
      shard_empty_kernel<false><<<grid, 256, 0, stream>>>(mode, static_cast<int>(M), scale, sh);
    return cudaGetLastError();
  }
  const float inv = block > 1 ? static_cast<float>(1.0 / sqrt(static_cast<double>(block))) : 1.0f;
  const int k = static_cast<int>(Ns);
#define B2_SQ(DT, F)                                                                                        \
  return mode == kLaneAmax                                                                                  \
             ? launch_lane<DT, F, kLaneAmax>(M, stream, y, ldy, k, block, inv, nullptr, ldq, scale, 0, sh)  \
         : mode == kLaneCodes                                                                               \
             ? launch_lane<DT, F, kLaneCodes>(M, stream, y, ldy, k, block, inv, nullptr, ldq, scale, 0, sh) \
             : launch_lane<DT, F, kLaneFused>(M, stream, y, ldy, k, block, inv, nullptr, ldq, scale, 0, sh)
#define B2_SQ_DT(F)                  \
  switch (y_dtype) {                 \
    case kF32: B2_SQ(kF32, F);       \
    case kF16: B2_SQ(kF16, F);       \
    case kBF16: B2_SQ(kBF16, F);     \
    default: return cudaErrorInvalidValue; \
  }
  if (quant == 1) { B2_SQ_DT(true) }
  B2_SQ_DT(false)
#undef B2_SQ_DT
#undef B2_SQ
}

// fp8 (e4m3fn / e5m2) -> fp32 / fp16 decode, exact for every finite pattern;
// NaN and infinity classes preserved (reference _decode_bits /
// _decode_weight, rdna2_ops/fp8_weight_gemm_v06.py:22-46).
__global__ void fp8_decode_kernel(const uint8_t* __restrict__ w, int fp8_dtype, int64_t rows, int64_t cols,
                                  int64_t ld, int out_dtype, void* __restrict__ out, int64_t ldo) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * cols) return;
  const int64_t r = i / cols, c = i % cols;
  const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(w[r * ld + c]),
                                               fp8_dtype == kE4M3 ? __NV_E4M3 : __NV_E5M2);
  if (out_dtype == kF16) static_cast<__half_raw*>(out)[r * ldo + c] = h;
  else static_cast<float*>(out)[r * ldo + c] = __half2float(__half(h));
}

cudaError_t run_fp8_decode(const void* w, int fp8_dtype, int64_t rows, int64_t cols, int64_t ld,
                           int out_dtype, void* out, int64_t ldo, cudaStream_t stream) {
  const int64_t total = rows * cols;
  if (total == 0) return cudaSuccess;
  fp8_decode_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(
      static_cast<const uint8_t*>(w), fp8_dtype, rows, cols, ld, out_dtype, out, ldo);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ repack

template <typename T>
__global__ void repack_kernel(const T* __restrict__ src, int64_t rows, int64_t cols, int64_t s_row,
                              int64_t s_col, T* __restrict__ dst, int64_t ldd, int row_fast) {
  __shared__ T tile[32][33];
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 32, c0 = static_cast<int64_t>(blockIdx.x) * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int64_t r = row_fast ? r0 + threadIdx.x : r0 + i;
    const int64_t c = row_fast ? c0 + i : c0 + threadIdx.x;
    T val = T(0);
    if (r < rows && c < cols) val = src[r * s_row + c * s_col];
    if (row_fast) tile[threadIdx.x][i] = val;
    else tile[i][threadIdx.x] = val;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int64_t r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < ldd) dst[r * ldd + c] = tile[i][threadIdx.x];
  }
}

cudaError_t run_repack(const void* src, int elem_bytes, int64_t rows, int64_t cols, int64_t s_row,
                       int64_t s_col, void* dst, int64_t ldd, cudaStream_t stream) {
  if (rows == 0 || ldd == 0) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>((ldd + 31) / 32), static_cast<unsigned>((rows + 31) / 32));
  if (grid.y > 65535u) return cudaErrorInvalidValue;
  const dim3 block(32, 8);
  const int row_fast = (s_row < 0 ? -s_row : s_row) < (s_col < 0 ? -s_col : s_col);
  if (elem_bytes == 1)
    repack_kernel<uint8_t><<<grid, block, 0, stream>>>(static_cast<const uint8_t*>(src), rows, cols,
                                                       s_row, s_col, static_cast<uint8_t*>(dst), ldd,
                                                       row_fast);
  else if (elem_bytes == 2)
    repack_kernel<uint16_t><<<grid, block, 0, stream>>>(static_cast<const uint16_t*>(src), rows, cols,
                                                        s_row, s_col, static_cast<uint16_t*>(dst), ldd,
                                                        row_fast);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace b2
