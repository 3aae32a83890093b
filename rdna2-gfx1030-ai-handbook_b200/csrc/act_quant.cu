// Activation prologue for sm_100a: optional orthonormal block-Hadamard
// rotation, per-row absmax and round-to-nearest-even quantization to INT8
// (scale = absmax/127) or e4m3 (scale = absmax/448), one pass over HBM.
//
// Replaces the Kitchen ConvRot + quantize_int8_rowwise pair called at
// production/MOSS_RDNA2_INT8/backend.py:112-122 and the row quantizer
// _quant_rows of rdna2_ops/fp8_weight_gemm_v06.py:76-92 (ties to even here).
//
// Layout: a row is split into 256-element segments; lane l of a warp holds
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

template <int DT>
__device__ __forceinline__ void load8(const void* x, int64_t off, bool vec, int valid, float (&v)[8]) {
  if (vec && valid == 8) {
    if constexpr (DT == kF32) {
      const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(x) + off);
      const float4 a = __ldg(p), b = __ldg(p + 1);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + off));
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
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
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = j < valid ? load_as_float(x, DT, off + j) : 0.0f;
  }
}

template <int QUANT>
__device__ __forceinline__ uint32_t encode(float v, float s) {
  const float z = __fdiv_rn(v, s);
  if constexpr (QUANT == 0) {
    int q = __float2int_rn(z);
    q = q > 127 ? 127 : (q < -127 ? -127 : q);
    return static_cast<uint32_t>(q) & 0xffu;
  } else {
    return static_cast<uint32_t>(__nv_cvt_float_to_fp8(z, __NV_SATFINITE, __NV_E4M3));
  }
}

template <int DT, int SPW, int QUANT>
__global__ void __launch_bounds__(128)
    act_quant_kernel(const void* __restrict__ x, int64_t ldx, int M, int K, int wpr, int block,
                     float inv, uint8_t* __restrict__ q, int64_t ldq, float* __restrict__ scale,
                     int vec_in, int vec_out) {
  __shared__ float s_max[4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * (4 / wpr) + warp / wpr;
  const int part = warp % wpr;
  const bool live = row < M;
  const int64_t seg0 = static_cast<int64_t>(part) * SPW;

  float v[SPW][8];
#pragma unroll
  for (int s = 0; s < SPW; ++s) {
    const int64_t k0 = (seg0 + s) * 256 + lane * 8;
    int64_t rem = static_cast<int64_t>(K) - k0;
    const int valid = live ? static_cast<int>(rem < 0 ? 0 : (rem > 8 ? 8 : rem)) : 0;
    load8<DT>(x, live ? static_cast<int64_t>(row) * ldx + k0 : 0, vec_in != 0, valid, v[s]);
  }

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
        const bool upper = (lane & d) != 0;
#pragma unroll
        for (int s = 0; s < SPW; ++s)
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float o = __shfl_xor_sync(0xffffffffu, v[s][i], d);
            v[s][i] = upper ? __fsub_rn(o, v[s][i]) : __fadd_rn(v[s][i], o);
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
    if (lane == 0) s_max[warp] = amax;
    __syncthreads();
    const int first = (warp / wpr) * wpr;
    for (int w = 0; w < wpr; ++w) amax = fmaxf(amax, s_max[first + w]);
  }
  float sc = __fdiv_rn(amax, QUANT == 0 ? 127.0f : 448.0f);
  if (!(sc > 0.0f)) sc = 1.0f;
  if (!live) return;

#pragma unroll
  for (int s = 0; s < SPW; ++s) {
    const int64_t k0 = (seg0 + s) * 256 + lane * 8;
    if (k0 >= K) continue;
    uint8_t* dst = q + static_cast<int64_t>(row) * ldq + k0;
    if (vec_out && k0 + 8 <= K) {
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        lo |= encode<QUANT>(v[s][i], sc) << (8 * i);
        hi |= encode<QUANT>(v[s][i + 4], sc) << (8 * i);
      }
      *reinterpret_cast<uint2*>(dst) = make_uint2(lo, hi);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (k0 + i < K) dst[i] = static_cast<uint8_t>(encode<QUANT>(v[s][i], sc));
    }
  }
  if (part == 0 && lane == 0) scale[row] = sc;
}

template <int DT, int QUANT>
static cudaError_t launch_spw(int spw, dim3 grid, cudaStream_t st, const void* x, int64_t ldx, int M,
                             int K, int wpr, int block, float inv, uint8_t* q, int64_t ldq,
                             float* scale, int vin, int vout) {
#define B2_SPW_CASE(S)                                                                          \
  case S:                                                                                       \
    act_quant_kernel<DT, S, QUANT><<<grid, 128, 0, st>>>(x, ldx, M, K, wpr, block, inv, q, ldq, \
                                                          scale, vin, vout);                    \
    break;
  switch (spw) {
    B2_SPW_CASE(1) B2_SPW_CASE(2) B2_SPW_CASE(3) B2_SPW_CASE(4) B2_SPW_CASE(5) B2_SPW_CASE(6)
    B2_SPW_CASE(7) B2_SPW_CASE(8) B2_SPW_CASE(10) B2_SPW_CASE(12) B2_SPW_CASE(16)
    default: return cudaErrorInvalidValue;
  }
#undef B2_SPW_CASE
  return cudaGetLastError();
}

// Pick warps-per-row and segments-per-warp: fewest warps whose registers hold
// the row, with warp ranges aligned to the rotation block.
static bool choose_layout(int64_t K, int block, int* wpr, int* spw) {
  // Up to 12 segments (96 fp32 values) per lane stay in registers without
  // spilling; 16 is the last resort for 12288 < K <= 16384.
  static const int kSpw[] = {1, 2, 3, 4, 5, 6, 7, 8, 10, 12};
  for (int w : {1, 2, 4, 5}) {
    if (w == 5) {
      if (K > 4 * 16 * 256 || (block > 1 && (block > 16 * 256 || (16 * 256) % block != 0))) return false;
      *wpr = 4;
      *spw = 16;
      return true;
    }
    for (int s : kSpw) {
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
                          int quant, void* q, int64_t ldq, float* scale, cudaStream_t stream) {
  if (M == 0) return cudaSuccess;
  int wpr = 1, spw = 1;
  if (!choose_layout(K, block, &wpr, &spw)) return cudaErrorInvalidValue;
  const int eb = x_dtype == kF32 ? 4 : 2;
  const int vin = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && ((ldx * eb) % 16 == 0);
  const int vout = (reinterpret_cast<uintptr_t>(q) % 8 == 0) && (ldq % 8 == 0);
  const float inv = block > 1 ? static_cast<float>(1.0 / sqrt(static_cast<double>(block))) : 1.0f;
  const int rows_per_cta = 4 / wpr;
  const dim3 grid(static_cast<unsigned>((M + rows_per_cta - 1) / rows_per_cta));
  uint8_t* qb = static_cast<uint8_t*>(q);
  const int m = static_cast<int>(M), k = static_cast<int>(K);
  if (quant == 0) {
    if (x_dtype == kF32) return launch_spw<kF32, 0>(spw, grid, stream, x, ldx, m, k, wpr, block, inv, qb, ldq, scale, vin, vout);
    if (x_dtype == kF16) return launch_spw<kF16, 0>(spw, grid, stream, x, ldx, m, k, wpr, block, inv, qb, ldq, scale, vin, vout);
    return launch_spw<kBF16, 0>(spw, grid, stream, x, ldx, m, k, wpr, block, inv, qb, ldq, scale, vin, vout);
  }
  if (x_dtype == kF32) return launch_spw<kF32, 1>(spw, grid, stream, x, ldx, m, k, wpr, block, inv, qb, ldq, scale, vin, vout);
  if (x_dtype == kF16) return launch_spw<kF16, 1>(spw, grid, stream, x, ldx, m, k, wpr, block, inv, qb, ldq, scale, vin, vout);
  return launch_spw<kBF16, 1>(spw, grid, stream, x, ldx, m, k, wpr, block, inv, qb, ldq, scale, vin, vout);
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
