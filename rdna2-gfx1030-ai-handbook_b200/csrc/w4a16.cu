// W4A16 weight-only GEMM for sm_100a: y[m,n] = sum_k a[m,k] * w[n,k] (+bias[n]),
// with w[n,k] = round_to_half((u[n,k] - zu[n,g]) * s[n,g]), g = k / group.
//
// Replaces int4_linear_a16 / _linear_dot2 of the reference
// (rdna2_ops/int4_weight_gemm_v07.py:540-564, 365-387), which decodes each
// weight as ((q - z).to(fp32) * s).to(fp16) inside the K loop and
// accumulates fp16 x fp16 products in fp32.
//
// Weight format (the north-star uint4 layout, nibbles interleaved for the
// kernel): eight unsigned nibbles per 32-bit word, word k/8 of its row
// ([N, K/8]); element j = k % 8 sits at nibble position (j >> 1) + 4 * (j & 1),
// so masking nibbles {i, i+4} yields elements (2i, 2i+1) in K order.  Scales
// and zero points are [N, K/group] in the activation's 16-bit type (zero
// points are the integers zu in [0,15]).  The reference's PackedInt4 stores
// signed nibbles q = u - 8 in natural order and zeros zu - 8; the value
// q - z = u - zu is the same, and b2_int4_to_w4a16_words converts the words.
//
// B200 design: swap-AB.  The dequantized weight tile is the 128-row A operand
// of tcgen05.mma kind::f16 and the tokens are its N dimension (32..256), so
// the same kernel serves decode (M = 1..16) and prefill (M = 2048).  Per
// 64-element k-block: warp 0 TMA-loads the packed words (4 KiB) and the
// activation tile (SW128); warps 2..5 unpack nibbles in registers
// (0x4300 | u is bf16 128+u, 0x6400 | u is fp16 1024+u), subtract the zero
// point exactly and multiply by the scale with one rounding, and store the
// 16-bit weights straight into the 128B-swizzled K-major layout the MMA
// reads; warp 1 issues 4 MMAs (K = 16 each) per k-block into a 128 x BT fp32
// TMEM accumulator.  Small M splits K across CTAs; a second kernel sums the
// fp32 partials in a fixed order, so results are run-to-run deterministic.
#include "b2_common.cuh"
#include "b2_internal.h"

namespace b2 {

struct W4Params {
  int M, N, K, group;
  const uint32_t* wq;      // [N, K/8] packed nibbles
  int64_t ldw;             // words per weight row
  const uint16_t* scales;  // [N, K/group]
  const uint16_t* zeros;   // [N, K/group]
  int64_t ldsz;            // elements per scales/zeros row
  const void* bias;        // [N] or nullptr
  int bias_dtype;
  void* out;               // [M, N] in the activation dtype (splits == 1)
  int64_t ldo;
  float* partial;          // [splits, M, N] fp32 (splits > 1)
  int splits, kb_per_split, num_kb, tiles_t;
  int stage_groups;        // groups staged in shared memory per CTA (>= groups of a split)
  int* status;
};

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// One 32-bit word of 8 interleaved nibbles -> 8 16-bit weights (one 16-byte
// chunk) in K order.
template <bool BF16>
__device__ __forceinline__ uint4 dequant_word(uint32_t w, uint32_t zz, uint32_t ss) {
  constexpr uint32_t kBias = BF16 ? 0x43004300u : 0x64006400u;  // 128+u (bf16), 1024+u (fp16)
  uint32_t r[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t t = ((w >> (4 * i)) & 0x000F000Fu) | kBias;   // elements (2i, 2i+1)
    if constexpr (BF16) {
      // (128+u) - (128+zu) is exact; one rounding in the product.
      const __nv_bfloat162 d = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&t),
                                       *reinterpret_cast<const __nv_bfloat162*>(&zz));
      const __nv_bfloat162 v = __hmul2(d, *reinterpret_cast<const __nv_bfloat162*>(&ss));
      r[i] = *reinterpret_cast<const uint32_t*>(&v);
    } else {
      const __half2 d = __hsub2(*reinterpret_cast<const __half2*>(&t),
                                *reinterpret_cast<const __half2*>(&zz));
      const __half2 v = __hmul2(d, *reinterpret_cast<const __half2*>(&ss));
      r[i] = *reinterpret_cast<const uint32_t*>(&v);
    }
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

// Per-(row, group) operands of dequant_word: {128+zu, 128+zu} and {s, s}.
template <bool BF16>
__device__ __forceinline__ void group_operands(const W4Params& p, int n, int g, uint32_t& zz,
                                               uint32_t& ss) {
  uint16_t s = 0, z = 0;
  if (n < p.N) {
    s = p.scales[static_cast<int64_t>(n) * p.ldsz + g];
    z = p.zeros[static_cast<int64_t>(n) * p.ldsz + g];
  }
  uint16_t zb;
  if constexpr (BF16) {
    const float zf = __bfloat162float(__ushort_as_bfloat16(z)) + 128.0f;  // exact integer
    zb = __bfloat16_as_ushort(__float2bfloat16_rn(zf));
  } else {
    const float zf = __half2float(__ushort_as_half(z)) + 1024.0f;
    zb = __half_as_ushort(__float2half_rn(zf));
  }
  zz = static_cast<uint32_t>(zb) | (static_cast<uint32_t>(zb) << 16);
  ss = static_cast<uint32_t>(s) | (static_cast<uint32_t>(s) << 16);
}

template <int BT, int STAGES>
struct W4Smem {
  static constexpr int kXfBytes = 128 * 128;          // dequantized weights, SW128
  static constexpr int kActBytes = BT * 128;          // activation tile, SW128
  static constexpr int kRawBytes = 128 * 32;          // packed words
  static constexpr int kStageBytes = kXfBytes + kActBytes + kRawBytes;
  static constexpr int kOffXf = 0;
  static constexpr int kOffAct = STAGES * kXfBytes;
  static constexpr int kOffRaw = kOffAct + STAGES * kActBytes;
  static constexpr int kOffBar = kOffRaw + STAGES * kRawBytes;
  static constexpr int kNumBars = 3 * STAGES + 1;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kOffGroups = kOffMisc + 16;     // [2][128][stage_groups] u32, dynamic
  static constexpr int kFixed = kOffGroups + 1024;     // + group staging at launch
  static constexpr uint32_t kTmemCols = BT < 32 ? 32 : BT;
  static constexpr int kMaxGroups = (232448 - kFixed) / (2 * 128 * 4);
  static_assert(kMaxGroups >= 8, "shared memory budget");
};

constexpr int kW4Threads = 320;  // producer, MMA, 8 transform warps (4 of them also epilogue)

template <bool BF16, int BT, int STAGES>
__global__ void __launch_bounds__(kW4Threads, 1)
    w4a16_kernel(const __grid_constant__ CUtensorMap tma_w, const __grid_constant__ CUtensorMap tma_a,
                 const W4Params p) {
  using L = W4Smem<BT, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint64_t* full_raw = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* full_xf = full_raw + STAGES;
  uint64_t* empty = full_xf + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // blockIdx.x: weight tile (128 rows of N); blockIdx.y: token tile; blockIdx.z: K split
  const int n0 = blockIdx.x * 128;
  const int t0 = blockIdx.y * BT;
  const int split = blockIdx.z;
  const int kb0 = split * p.kb_per_split;
  int kb1 = kb0 + p.kb_per_split;
  if (kb1 > p.num_kb) kb1 = p.num_kb;
  const int nkb = kb1 > kb0 ? kb1 - kb0 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_raw[s], 1);
      mbar_init(&full_xf[s], 8);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&tfull[0], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tma_w);
    tma_prefetch_desc(&tma_a);
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
      for (int i = 0; i < nkb; ++i) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kSiteProducer, p.status)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full_raw[stage], L::kRawBytes + L::kActBytes);
        const int kb = kb0 + i;
        tma_load_2d(&tma_w, &full_raw[stage], smem + L::kOffRaw + stage * L::kRawBytes, kb * 8, n0);
        tma_load_2d(&tma_a, &full_raw[stage], smem + L::kOffAct + stage * L::kActBytes, kb * 64, t0);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      for (int i = 0; i < STAGES && ok; ++i) {  // tail: all slots released
        ok = mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kSiteProducer, p.status);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = (1u << 4) | (BF16 ? (1u << 7) | (1u << 10) : 0u) |
                                 (static_cast<uint32_t>(BT >> 3) << 17) | (static_cast<uint32_t>(128 >> 4) << 24);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int i = 0; i < nkb; ++i) {
        if (!mbar_wait(&full_xf[stage], phase, abort_flag, kSiteMma, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + L::kOffXf + stage * L::kXfBytes);
        const uint32_t b_addr = smem_u32(smem + L::kOffAct + stage * L::kActBytes);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma<kKindBF16>(tmem_base, sw128_desc(a_addr + kk * 32), sw128_desc(b_addr + kk * 32), idesc,
                          (i | kk) != 0 ? 1u : 0u);
        umma_commit(&empty[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) umma_commit(&tfull[0]);
    }
  } else {
    // ---- transform: 256 threads; thread (r, h) dequantizes words 4h..4h+3
    // (elements 32h..32h+31) of weight row n0 + r of every k-block.
    const int t = threadIdx.x - 64;  // 0..255
    const int r = t & 127, h = t >> 7;
    const int n = n0 + r;
    const int g_first = (kb0 * 64) / p.group;
    const int ng = p.stage_groups;
    uint32_t* s_zz = reinterpret_cast<uint32_t*>(smem + L::kOffGroups);
    uint32_t* s_ss = s_zz + 128 * ng;
    // Stage this CTA's (128 rows x ng groups) zero/scale operands once.
    for (int i = t; i < 128 * ng; i += 256) {
      const int rr = i / ng, gg = i % ng;
      const int g = g_first + gg;
      uint32_t zz = 0, ss = 0;
      if (g < p.K / p.group) group_operands<BF16>(p, n0 + rr, g, zz, ss);
      s_zz[rr * ng + gg] = zz;
      s_ss[rr * ng + gg] = ss;
    }
    named_bar_sync(1, 256);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int i = 0; i < nkb && ok; ++i) {
      const int kb = kb0 + i;
      const int gl = (kb * 64 + h * 32) / p.group - g_first;  // 32 elements never straddle a group
      const uint32_t zz = s_zz[r * ng + gl], ss = s_ss[r * ng + gl];
      ok = mbar_wait(&full_raw[stage], phase, abort_flag, kSiteTransform, p.status);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      const uint4 w = *reinterpret_cast<const uint4*>(smem + L::kOffRaw + stage * L::kRawBytes + r * 32 + h * 16);
      const uint32_t words[4] = {w.x, w.y, w.z, w.w};
      uint8_t* xf = smem + L::kOffXf + stage * L::kXfBytes + r * 128;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = 4 * h + j;
        *reinterpret_cast<uint4*>(xf + ((c ^ (r & 7)) << 4)) = dequant_word<BF16>(words[j], zz, ss);
      }
      fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(&full_xf[stage]);
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
    (void)n;
    // ---- epilogue: TMEM lane = weight row, column = token
    if (ok && nkb > 0 && warp < 6) {
      const int quarter = warp & 3;
      bool done = mbar_wait(&tfull[0], 0, abort_flag, kSiteEpilogue, p.status);
      done = __all_sync(0xffffffffu, done);
      if (done) {
        tc_fence_after();
        const int row = n0 + quarter * 32 + lane;  // output channel
        float bias = 0.0f;
        if (p.splits == 1 && p.bias != nullptr && row < p.N) bias = load_as_float(p.bias, p.bias_dtype, row);
#pragma unroll 1
        for (int c = 0; c < BT / 32; ++c) {
          uint32_t v[32];
          __syncwarp();
          tmem_ld32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(c * 32), v);
          tmem_ld_wait(v);
          if (row < p.N) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int m = t0 + c * 32 + j;
              if (m < p.M) {
                const float acc = __uint_as_float(v[j]);
                if (p.splits > 1) {
                  p.partial[(static_cast<int64_t>(split) * p.M + m) * p.N + row] = acc;
                } else {
                  const float y = __fadd_rn(acc, bias);
                  uint16_t* o = static_cast<uint16_t*>(p.out) + static_cast<int64_t>(m) * p.ldo + row;
                  *o = BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(y))
                            : __half_as_ushort(__float2half_rn(y));
                }
              }
            }
          }
        }
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

// out[m,n] = cast(sum_s partial[s,m,n] + bias[n]), s in increasing order.
template <bool BF16>
__global__ void splitk_reduce_kernel(const float* __restrict__ partial, int splits, int M, int N,
                                     const void* bias, int bias_dtype, void* out, int64_t ldo) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(M) * N) return;
  const int m = static_cast<int>(i / N), n = static_cast<int>(i % N);
  float acc = 0.0f;
  for (int s = 0; s < splits; ++s) acc = __fadd_rn(acc, partial[static_cast<int64_t>(s) * M * N + i]);
  if (bias != nullptr) acc = __fadd_rn(acc, load_as_float(bias, bias_dtype, n));
  uint16_t* o = static_cast<uint16_t*>(out) + static_cast<int64_t>(m) * ldo + n;
  *o = BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(acc)) : __half_as_ushort(__float2half_rn(acc));
}

// Reference PackedInt4 words (signed nibbles q = u - 8, element j at nibble
// j) -> kernel words (unsigned nibbles u, element j at nibble
// (j >> 1) + 4 * (j & 1)).
__global__ void w4a16_words_kernel(const uint32_t* __restrict__ src, uint32_t* __restrict__ dst, int64_t n) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t u = src[i] ^ 0x88888888u;
  uint32_t w = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) w |= ((u >> (4 * j)) & 15u) << (4 * ((j >> 1) + 4 * (j & 1)));
  dst[i] = w;
}

// Group INT4 packer, one thread per (row, group): the restated semantics of
// the reference's pack_int4 / _pack_weight (rdna2_ops/int4_weight_gemm_v07.py
// :103-137, 413-430): IEEE divisions, round-half-even, signed nibbles
// q - 8 (affine) or q (symmetric), fp32 scales, int32 zeros (zu - 8), sums.
// w: [N, K] of w_dtype (0 f32, 1 f16, 2 bf16) with row stride ldw_el.
// data: layout 0 = "nk" [N, K/8] words, 1 = "kn" [K/8, N]; order_high puts
// element 0 in the top nibble.
__global__ void pack_int4_kernel(const void* __restrict__ w, int w_dtype, int64_t ldw_el, int N, int K,
                                 int G, int symmetric, int layout_kn, int order_high,
                                 int32_t* __restrict__ data, float* __restrict__ scales,
                                 int32_t* __restrict__ zeros, int32_t* __restrict__ sums) {
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int ng = K / G;
  if (gid >= static_cast<int64_t>(N) * ng) return;
  const int n = static_cast<int>(gid / ng), g = static_cast<int>(gid % ng);
  const int64_t base = static_cast<int64_t>(n) * ldw_el + static_cast<int64_t>(g) * G;
  float scale;
  int zu = 0, zero = 0;
  bool empty = false;
  if (symmetric) {
    float amax = 0.0f;
    for (int i = 0; i < G; ++i) amax = fmaxf(amax, fabsf(load_as_float(w, w_dtype, base + i)));
    scale = __fdiv_rn(amax, 7.0f);
    if (scale == 0.0f) scale = 1.0f;
  } else {
    float lo = 0.0f, hi = 0.0f;
    for (int i = 0; i < G; ++i) {
      const float x = load_as_float(w, w_dtype, base + i);
      lo = fminf(lo, x);
      hi = fmaxf(hi, x);
    }
    scale = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
    empty = scale == 0.0f;
    if (empty) scale = 1.0f;
    float z = rintf(__fdiv_rn(-lo, scale));
    z = fminf(fmaxf(z, 0.0f), 15.0f);
    zu = static_cast<int>(z);
    zero = empty ? 0 : zu - 8;
  }
  int total = 0;
  for (int w8 = 0; w8 < G / 8; ++w8) {
    uint32_t word = 0;
    for (int j = 0; j < 8; ++j) {
      const float x = load_as_float(w, w_dtype, base + w8 * 8 + j);
      int q;
      if (symmetric) {
        q = static_cast<int>(fminf(fmaxf(rintf(__fdiv_rn(x, scale)), -7.0f), 7.0f));
      } else {
        const float u = fminf(fmaxf(__fadd_rn(rintf(__fdiv_rn(x, scale)), static_cast<float>(zu)), 0.0f), 15.0f);
        q = empty ? 0 : static_cast<int>(u) - 8;
      }
      total += q;
      const int shift = order_high ? 28 - 4 * j : 4 * j;
      word |= (static_cast<uint32_t>(q) & 15u) << shift;
    }
    const int64_t kw = static_cast<int64_t>(g) * (G / 8) + w8;
    if (layout_kn) data[kw * N + n] = static_cast<int32_t>(word);
    else data[static_cast<int64_t>(n) * (K / 8) + kw] = static_cast<int32_t>(word);
  }
  scales[static_cast<int64_t>(n) * ng + g] = scale;
  zeros[static_cast<int64_t>(n) * ng + g] = zero;
  sums[static_cast<int64_t>(n) * ng + g] = total;
}

// Decode packed signed nibbles to integers (q - z) or values (q - z) * s:
// the reference's unpack_int4 / _unpack_weight (int4_weight_gemm_v07.py:
// 139-152, 433-441).  out_dtype 0 f32, 1 f16, 3 int8 (integer mode).
__global__ void unpack_int4_kernel(const int32_t* __restrict__ data, int layout_kn, int order_high,
                                   const float* __restrict__ scales, const int32_t* __restrict__ zeros,
                                   int N, int K, int G, int out_dtype, void* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(N) * K) return;
  const int n = static_cast<int>(i / K), k = static_cast<int>(i % K);
  const uint32_t word = static_cast<uint32_t>(
      layout_kn ? data[static_cast<int64_t>(k / 8) * N + n] : data[static_cast<int64_t>(n) * (K / 8) + k / 8]);
  const int shift = order_high ? 28 - 4 * (k % 8) : 4 * (k % 8);
  int q = static_cast<int>((word >> shift) & 15u);
  if (q >= 8) q -= 16;
  const int64_t gi = static_cast<int64_t>(n) * (K / G) + k / G;
  const int v = q - zeros[gi];
  if (out_dtype == 3) {
    static_cast<int8_t*>(out)[i] = static_cast<int8_t>(v);
  } else {
    const float f = __fmul_rn(static_cast<float>(v), scales[gi]);
    if (out_dtype == kF32) static_cast<float*>(out)[i] = f;
    else static_cast<__half*>(out)[i] = __float2half_rn(f);
  }
}

// ----------------------------------------------------------------- host
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn tensor_map_encoder();

static cudaError_t map_2d(CUtensorMap* map, const void* ptr, CUtensorMapDataType dt, int elem_bytes,
                          int64_t inner, int64_t rows, int64_t stride_bytes, uint32_t box_inner,
                          uint32_t box_rows, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = tensor_map_encoder();
  if (fn == nullptr) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(stride_bytes)};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  (void)elem_bytes;
  CUresult r = fn(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <bool BF16, int BT, int STAGES>
static cudaError_t launch_w4(const void* a, int64_t lda, W4Params p, cudaStream_t stream) {
  using L = W4Smem<BT, STAGES>;
  auto kernel = w4a16_kernel<BF16, BT, STAGES>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return cudaErrorInvalidDevice;
  if (p.stage_groups > L::kMaxGroups) return cudaErrorInvalidValue;
  const int smem = L::kFixed + 2 * 128 * 4 * p.stage_groups;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         L::kFixed + 2 * 128 * 4 * L::kMaxGroups);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  CUtensorMap mw, ma;
  cudaError_t e = map_2d(&mw, p.wq, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, p.K / 8, p.N, p.ldw * 4, 8, 128,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
  if (e != cudaSuccess) return e;
  e = map_2d(&ma, a, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, p.K, p.M, lda * 2, 64, BT,
             CU_TENSOR_MAP_SWIZZLE_128B);
  if (e != cudaSuccess) return e;
  p.tiles_t = (p.M + BT - 1) / BT;
  dim3 grid((p.N + 127) / 128, p.tiles_t, p.splits);
  kernel<<<grid, kW4Threads, smem, stream>>>(mw, ma, p);
  return cudaGetLastError();
}

// Token tile for M tokens (each with its own ring depth below).
static int w4_bt(int64_t M) { return M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256; }
static int w4_max_groups(int bt) {
  return bt == 32 ? W4Smem<32, 4>::kMaxGroups : bt == 64 ? W4Smem<64, 6>::kMaxGroups
       : bt == 128 ? W4Smem<128, 5>::kMaxGroups : W4Smem<256, 3>::kMaxGroups;
}

// Split count and staged groups per CTA: fill the machine for small token
// counts (at least 4 k-blocks per split) and keep a split's scale/zero
// operands within the shared-memory staging area.
void w4a16_plan(int64_t M, int64_t N, int64_t K, int group, int* splits_out, int* kbps_out,
                int* groups_out) {
  const int bt = w4_bt(M);
  const int64_t num_kb = K / 64;
  const int64_t ctas = ((N + 127) / 128) * ((M + bt - 1) / bt);
  int64_t s = (2 * static_cast<int64_t>(device_sm_count()) + ctas - 1) / ctas;
  const int64_t max_s = num_kb / 4 > 0 ? num_kb / 4 : 1;
  if (s > max_s) s = max_s;
  if (s < 1) s = 1;
  for (;;) {
    const int64_t kbps = (num_kb + s - 1) / s;
    const int64_t groups = kbps * 64 / group + 2;
    if (groups <= w4_max_groups(bt) || s >= num_kb) {
      *splits_out = static_cast<int>((num_kb + kbps - 1) / kbps);
      *kbps_out = static_cast<int>(kbps);
      *groups_out = static_cast<int>(groups);
      return;
    }
    ++s;
  }
}

cudaError_t run_w4a16(const void* a, int a_dtype, int64_t lda, const uint32_t* wq, int64_t ldw,
                      const uint16_t* scales, const uint16_t* zeros, int64_t ldsz, int group,
                      int64_t M, int64_t N, int64_t K, const void* bias, int bias_dtype, void* out,
                      int64_t ldo, float* partial, size_t partial_bytes, cudaStream_t stream) {
  if (M == 0 || N == 0) return cudaSuccess;
  W4Params p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.group = group;
  p.wq = wq;
  p.ldw = ldw;
  p.scales = scales;
  p.zeros = zeros;
  p.ldsz = ldsz;
  p.bias = bias;
  p.bias_dtype = bias_dtype;
  p.out = out;
  p.ldo = ldo;
  p.num_kb = static_cast<int>(K / 64);
  p.status = status_word_ptr();
  w4a16_plan(M, N, K, group, &p.splits, &p.kb_per_split, &p.stage_groups);
  if (p.splits > 1) {
    if (partial == nullptr || partial_bytes < static_cast<size_t>(p.splits) * M * N * 4)
      return cudaErrorInvalidValue;
    p.partial = partial;
  }
  const bool bf = a_dtype == kBF16;
  const int bt = w4_bt(M);
  cudaError_t e;
  if (bt == 32) e = bf ? launch_w4<true, 32, 4>(a, lda, p, stream) : launch_w4<false, 32, 4>(a, lda, p, stream);
  else if (bt == 64) e = bf ? launch_w4<true, 64, 6>(a, lda, p, stream) : launch_w4<false, 64, 6>(a, lda, p, stream);
  else if (bt == 128) e = bf ? launch_w4<true, 128, 5>(a, lda, p, stream) : launch_w4<false, 128, 5>(a, lda, p, stream);
  else e = bf ? launch_w4<true, 256, 3>(a, lda, p, stream) : launch_w4<false, 256, 3>(a, lda, p, stream);
  if (e != cudaSuccess || p.splits == 1) return e;
  const int64_t total = M * N;
  const unsigned blocks = static_cast<unsigned>((total + 255) / 256);
  if (bf) splitk_reduce_kernel<true><<<blocks, 256, 0, stream>>>(partial, p.splits, p.M, p.N, bias, bias_dtype, out, ldo);
  else splitk_reduce_kernel<false><<<blocks, 256, 0, stream>>>(partial, p.splits, p.M, p.N, bias, bias_dtype, out, ldo);
  return cudaGetLastError();
}

cudaError_t run_pack_int4(const void* w, int w_dtype, int64_t ldw_el, int64_t N, int64_t K, int G,
                          int symmetric, int layout_kn, int order_high, int32_t* data, float* scales,
                          int32_t* zeros, int32_t* sums, cudaStream_t stream) {
  const int64_t groups = N * (K / G);
  if (groups == 0) return cudaSuccess;
  pack_int4_kernel<<<static_cast<unsigned>((groups + 127) / 128), 128, 0, stream>>>(
      w, w_dtype, ldw_el, static_cast<int>(N), static_cast<int>(K), G, symmetric, layout_kn, order_high,
      data, scales, zeros, sums);
  return cudaGetLastError();
}

cudaError_t run_unpack_int4(const int32_t* data, int layout_kn, int order_high, const float* scales,
                            const int32_t* zeros, int64_t N, int64_t K, int G, int out_dtype, void* out,
                            cudaStream_t stream) {
  const int64_t total = N * K;
  if (total == 0) return cudaSuccess;
  unpack_int4_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(
      data, layout_kn, order_high, scales, zeros, static_cast<int>(N), static_cast<int>(K), G, out_dtype, out);
  return cudaGetLastError();
}

cudaError_t run_w4a16_words(const uint32_t* src, uint32_t* dst, int64_t n, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  w4a16_words_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(src, dst, n);
  return cudaGetLastError();
}

}  // namespace b2
