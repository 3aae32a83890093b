// W4A8 grouped linear for sm_100a: y[m,n] = (sum_g fp32(e_g[m,n]) * s[n,g]) * sa[m]
// (+ bias[n]), e_g = sum over group g of a[m,k] * (q[n,k] - z[n,g]) exactly;
// INTEGER mode returns sum_g e_g as int32.
//
// Replaces int4_linear_a8 and its _linear_dot4* kernels
// (rdna2_ops/int4_weight_gemm_v07.py:476-537, 182-217): per group an exact
// INT32 dot, times the fp32 group scale, accumulated in fp32 in group order
// (product and sum each rounded), then times the activation row scale and
// plus bias -- the order of grouped_integer_reference
// (int4_model_switches_v07.py:19-34), so outputs are bit-identical.
//
// B200 design: swap-AB tcgen05.mma kind::i8 -- the 128 weight rows of a tile
// are the A operand, the tokens (BT = 16, 32 or 64) are N.  The MMA runs on the
// raw nibbles u = q + 8 in [0, 15]; each group's accumulator is corrected
// exactly afterwards, e = acc_u - zu * asum (zu = z + 8, asum = the group's
// sum of a over its k, precomputed), which keeps the in-register unpack at
// a few logic ops per 16 weights.  A group's accumulator lives in its own
// TMEM columns; TMEM holds two k-blocks of group accumulators, so drain
// warps fold k-block kb into the fp32 totals while the MMA fills kb + 1.
//
// Weight format ("W4A8 tiles", b2_w4a8_prepare from PackedInt4):
//   tiles  u64 [T][K/128][8][128]: per (128-row tile, 128-element k-block),
//          word pair p of row r holds elements 16p..16p+15; inside each
//          32-bit half, element j sits at nibble 2j (j < 4) or 2(j - 4) + 1,
//          so w & 0x0F0F0F0F and (w >> 4) & 0x0F0F0F0F are the int8 bytes
//          in K order.  Word-pair-major rows make the shared loads
//          conflict-free.
//   groups u64 [T][K/group][128]: low half the fp32 scale, high half zu.
#include "b2_common.cuh"
#include "b2_internal.h"

namespace b2 {

constexpr int kW8Rows = 128;        // weight rows per tile (UMMA M)
constexpr int kW8Chunk = 8192;      // bytes of one (tile, k-block) of nibbles
constexpr int kW8MaxBT = 64;

struct W4A8Params {
  int M, N, K, group, T, KB, G, TM, P, integer;
  const uint64_t* groups;
  const uint8_t* tiles;
  const float* a_scale;
  const int32_t* asum;  // [G][Mp], Mp = round_up(M, 16), zero past M
  int Mp;
  const void* bias;
  int bias_dtype;
  void* out;            // fp32 or int32 [M, ldo]
  int64_t ldo;
  int* status;
};

template <int BT, int RK, int RS>
struct W8Layout {
  static constexpr int kXf = kW8Rows * 128;             // one k-block of int8 weights, SW128
  static constexpr int kAct = BT * 128;                 // BT tokens x 128 int8, SW128
  static constexpr int kWords = RK * kW8Chunk;
  static constexpr int kOffXf = 0;                      // 2 slots
  static constexpr int kOffAct = kOffXf + 2 * kXf;
  static constexpr int kOffWords = kOffAct + RS * RK * kAct;
  static constexpr int kOffBar = kOffWords + RS * kWords;
  static constexpr int kNumBars = 2 * RS + 4 + 4 + 1;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kAlloc = kOffMisc + 16 + 1024;
  static constexpr int kDrainWarps = 4 * (BT / 16);     // 16 token columns per drain thread
  static constexpr int kThreads = 32 * (2 + 8 + kDrainWarps);
  static_assert(kAlloc <= 232448, "shared memory budget");
  static_assert(kAct % 1024 == 0, "SW128 tiles need 1 KiB alignment");
};

__device__ __forceinline__ uint2 lds_v2u(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr) : "memory");
  return v;
}

template <int BT, int RK, int RS>
__global__ void __launch_bounds__(W8Layout<BT, RK, RS>::kThreads, 1)
    w4a8_kernel(const __grid_constant__ CUtensorMap tma_a, const W4A8Params p) {
  using L = W8Layout<BT, RK, RS>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint64_t* full_raw = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* raw_empty = full_raw + RS;
  uint64_t* full_xf = raw_empty + RS;   // [2]
  uint64_t* xf_empty = full_xf + 2;     // [2]
  uint64_t* acc_full = xf_empty + 2;    // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ngk = 128 / p.group;  // groups per k-block
  const uint32_t tcols = 2u * ngk * BT <= 32 ? 32u : 2u * ngk * BT <= 64 ? 64u : 2u * ngk * BT <= 128 ? 128u
                         : 2u * ngk * BT <= 256 ? 256u : 512u;
  const int num_tiles = p.T * p.TM;

  if (threadIdx.x == 0) {
    for (int s = 0; s < RS; ++s) {
      mbar_init(&full_raw[s], 1);
      mbar_init(&raw_empty[s], 8 + 1);  // transform warps + the MMA commit
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&full_xf[s], 4);
      mbar_init(&xf_empty[s], 1);
      mbar_init(&acc_full[s], 1);
      mbar_init(&acc_empty[s], L::kDrainWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tma_a);
  if (warp == 1) {
    tmem_alloc(tmem_slot, tcols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---- producer: packed nibbles (bulk copy) + activation tiles (TMA)
    int rs = 0;
    uint32_t rph = 0, live = 0, live_par = 0;
    bool ok = true;
    for (int x = blockIdx.x; x < num_tiles && ok; x += p.P) {
      const int tn = x / p.TM, tm = x % p.TM;
      for (int kb = 0; kb < p.KB; kb += RK) {
        const int n = p.KB - kb < RK ? p.KB - kb : RK;
        ok = __all_sync(0xffffffffu, mbar_wait(&raw_empty[rs], rph ^ 1u, abort_flag, kSiteProducer, p.status));
        if (!ok) break;
        if (elect_one()) {
          mbar_arrive_expect_tx(&full_raw[rs], static_cast<uint32_t>(n * (kW8Chunk + L::kAct)));
          bulk_load(smem + L::kOffWords + rs * L::kWords,
                    p.tiles + (static_cast<int64_t>(tn) * p.KB + kb) * kW8Chunk, n * kW8Chunk, &full_raw[rs]);
          for (int j = 0; j < n; ++j)
            tma_load_2d(&tma_a, &full_raw[rs], smem + L::kOffAct + (rs * RK + j) * L::kAct, (kb + j) * 128,
                        tm * BT);
        }
        __syncwarp();
        live |= 1u << rs;
        live_par = (live_par & ~(1u << rs)) | (rph << rs);
        if (++rs == RS) {
          rs = 0;
          rph ^= 1u;
        }
      }
    }
    for (int i = 0; i < RS && ok; ++i) {
      ok = __all_sync(0xffffffffu, mbar_wait(&raw_empty[rs], rph ^ 1u, abort_flag, kSiteProducer, p.status));
      if (++rs == RS) {
        rs = 0;
        rph ^= 1u;
      }
    }
    if (!ok && lane == 0) {
      const uint64_t t0 = globaltimer();
      for (int i = 0; i < RS; ++i)
        if ((live >> i) & 1u)
          while (!mbar_try_wait(&full_raw[i], (live_par >> i) & 1u) && globaltimer() - t0 < kWaitLimitNs) {
          }
    }
  } else if (warp == 1) {
    // ---- MMA issuer: 4 K=32 slices per k-block; a slice starting a group
    // overwrites that group's TMEM columns, the others accumulate.
    constexpr uint32_t idesc = make_idesc<kKindI8>(kW8Rows, BT);
    const uint64_t a_desc0 = sw128_desc(smem_u32(smem + L::kOffXf));
    const uint64_t b_desc0 = sw128_desc(smem_u32(smem + L::kOffAct));
    int rs = 0, xs = 0, kbi = 0;
    uint32_t xph = 0;
    bool ok = true;
    for (int x = blockIdx.x; x < num_tiles && ok; x += p.P) {
      for (int kb = 0; kb < p.KB && ok; kb += RK) {
        const int n = p.KB - kb < RK ? p.KB - kb : RK;
        for (int j = 0; j < n; ++j, ++kbi) {
          const int b = kbi & 1;
          ok = __all_sync(0xffffffffu, mbar_wait(&acc_empty[b], ((kbi >> 1) & 1) ^ 1u, abort_flag, kSiteMmaTmem,
                                                 p.status));
          if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&full_xf[xs], xph, abort_flag, kSiteMma, p.status));
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            const uint64_t ad = a_desc0 + static_cast<uint32_t>((xs * L::kXf) >> 4);
            const uint64_t bd = b_desc0 + static_cast<uint32_t>(((rs * RK + j) * L::kAct) >> 4);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const int gi = (kk * 32) / p.group;
              const bool first = (kk * 32) % p.group == 0;
              umma<kKindI8>(tmem_base + static_cast<uint32_t>((b * ngk + gi) * BT), ad + 2 * kk, bd + 2 * kk, idesc,
                            first ? 0u : 1u);
            }
            umma_commit(&xf_empty[xs]);
            umma_commit(&acc_full[b]);
          }
          __syncwarp();
          if (++xs == 2) {
            xs = 0;
            xph ^= 1u;
          }
        }
        if (!ok) break;
        if (elect_one()) umma_commit(&raw_empty[rs]);
        __syncwarp();
        if (++rs == RS) rs = 0;
      }
    }
    if (elect_one()) {
      umma_commit(drain);
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < kWaitLimitNs) {
      }
    }
    __syncwarp();
  } else if (warp < 10) {
    // ---- transform: 2 groups of 4 warps, k-block i into slot i % 2; one
    // thread per weight row unpacks 128 nibbles into 128 int8 bytes.
    const int t = threadIdx.x - 64;
    const int gi = t >> 7, r = t & 127;
    const uint32_t xrow = (smem_u32(smem + L::kOffXf + gi * L::kXf) + r * 128) | ((r & 7) << 4);
    int rs = 0, i = 0;
    uint32_t rph = 0, use = 0;
    bool ok = true;
    for (int x = blockIdx.x; x < num_tiles && ok; x += p.P) {
      for (int kb = 0; kb < p.KB; kb += RK) {
        const int n = p.KB - kb < RK ? p.KB - kb : RK;
        ok = __all_sync(0xffffffffu, mbar_wait(&full_raw[rs], rph, abort_flag, kSiteTransform, p.status));
        if (!ok) break;
        const uint32_t words = smem_u32(smem + L::kOffWords + rs * L::kWords) + r * 8;
        for (int j = 0; j < n; ++j, ++i) {
          if ((i & 1) != gi) continue;
          ok = __all_sync(0xffffffffu, mbar_wait(&xf_empty[gi], use ^ 1u, abort_flag, kSiteTransform, p.status));
          if (!ok) break;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const uint2 w = lds_v2u(words + j * kW8Chunk + q * kW8Rows * 8);
            sts_v4(xrow ^ (q << 4), make_uint4(w.x & 0x0F0F0F0Fu, (w.x >> 4) & 0x0F0F0F0Fu, w.y & 0x0F0F0F0Fu,
                                               (w.y >> 4) & 0x0F0F0F0Fu));
          }
          fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core
          __syncwarp();
          if (lane == 0) mbar_arrive(&full_xf[gi]);
          use ^= 1u;
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[rs]);
        if (++rs == RS) {
          rs = 0;
          rph ^= 1u;
        }
      }
    }
  } else {
    // ---- drain: warp (quarter q, column block cb) owns weight rows
    // q*32 + lane and token columns cb*16 .. cb*16 + 15 of the tile.
    const int dw = warp - 10;
    const int quarter = warp & 3, cb = dw >> 2;
    const int rt = quarter * 32 + lane;
    int kbi = 0;
    bool ok = true;
    for (int x = blockIdx.x; x < num_tiles && ok; x += p.P) {
      const int tn = x / p.TM, tm = x % p.TM;
      const int n = tn * kW8Rows + rt;
      const int m0 = tm * BT + cb * 16;
      float total[16];
      int32_t exact[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        total[j] = 0.0f;
        exact[j] = 0;
      }
      // Group operands run one group ahead of the accumulators: the loads for
      // group s + 1 are in flight while group s waits for and folds its TMEM
      // columns.  asum rows are padded to 16 tokens, so a thread's 16 sums are
      // four aligned 16-byte loads.
      const int total_groups = p.KB * ngk;
      auto fetch = [&](int gs, uint64_t& op, int4 (&as)[4]) {
        op = n < p.N ? __ldg(p.groups + (static_cast<int64_t>(tn) * p.G + gs) * kW8Rows + rt) : 0ull;
        const int4* src = reinterpret_cast<const int4*>(p.asum + static_cast<int64_t>(gs) * p.Mp + m0);
#pragma unroll
        for (int q = 0; q < 4; ++q) as[q] = __ldg(src + q);
      };
      uint64_t op_next;
      int4 as_next[4];
      fetch(0, op_next, as_next);
      int gs = 0;
      for (int kb = 0; kb < p.KB; ++kb, ++kbi) {
        const int b = kbi & 1;
        ok = __all_sync(0xffffffffu,
                        mbar_wait(&acc_full[b], (kbi >> 1) & 1, abort_flag, kSiteEpilogue, p.status));
        if (!ok) break;
        tc_fence_after();
        for (int gi = 0; gi < ngk; ++gi, ++gs) {
          const uint64_t op = op_next;
          const int4 a4[4] = {as_next[0], as_next[1], as_next[2], as_next[3]};
          if (gs + 1 < total_groups) fetch(gs + 1, op_next, as_next);
          const float s = __uint_as_float(static_cast<uint32_t>(op));
          const int32_t zu = static_cast<int32_t>(op >> 32);
          const int32_t as[16] = {a4[0].x, a4[0].y, a4[0].z, a4[0].w, a4[1].x, a4[1].y, a4[1].z, a4[1].w,
                                  a4[2].x, a4[2].y, a4[2].z, a4[2].w, a4[3].x, a4[3].y, a4[3].z, a4[3].w};
          uint32_t v[16];
          tmem_ld16(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                        static_cast<uint32_t>((b * ngk + gi) * BT + cb * 16),
                    v);
          tmem_ld_wait16(v);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int32_t e = static_cast<int32_t>(v[j]) - zu * as[j];
            if (p.integer) {
              exact[j] += e;
            } else {
              total[j] = __fadd_rn(total[j], __fmul_rn(static_cast<float>(e), s));
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[b]);
      }
      if (!ok) break;
      if (n < p.N) {
        const float bias = (!p.integer && p.bias != nullptr) ? load_as_float(p.bias, p.bias_dtype, n) : 0.0f;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = m0 + j;
          if (m < p.M) {
            if (p.integer) {
              static_cast<int32_t*>(p.out)[static_cast<int64_t>(m) * p.ldo + n] = exact[j];
            } else {
              float y = __fmul_rn(total[j], p.a_scale[m]);
              if (p.bias != nullptr) y = __fadd_rn(y, bias);
              static_cast<float*>(p.out)[static_cast<int64_t>(m) * p.ldo + n] = y;
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
    tmem_dealloc(tmem_base, tcols);
  }
}

// asum[g][m] = sum of a[m, k] over group g's k (exact int32); rows padded
// to Mp tokens with zeros.
__global__ void w4a8_asum_kernel(const int8_t* __restrict__ a, int64_t lda, int M, int Mp, int K, int group,
                                 int32_t* __restrict__ asum) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int G = K / group;
  if (i >= static_cast<int64_t>(Mp) * G) return;
  const int g = static_cast<int>(i / Mp), m = static_cast<int>(i % Mp);
  int32_t s = 0;
  if (m < M) {
    const int8_t* row = a + static_cast<int64_t>(m) * lda + static_cast<int64_t>(g) * group;
    for (int k = 0; k < group; ++k) s += row[k];
  }
  asum[i] = s;
}

// PackedInt4 words (signed nibbles q = u - 8, layout nk/kn, order low/high)
// -> W4A8 tiles; one thread per output 32-bit word (half of a word pair).
__global__ void w4a8_tiles_kernel(const uint32_t* __restrict__ data, int layout_kn, int order_high, int N, int K,
                                  int KB, int64_t total, uint32_t* __restrict__ tiles) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  // u32 index i -> (u64 index, half); u64 index = ((t*KB + kb)*8 + pair)*128 + r
  const int half = static_cast<int>(i & 1);
  const int64_t u = i >> 1;
  const int r = static_cast<int>(u & 127);
  const int pair = static_cast<int>((u >> 7) & 7);
  const int64_t rest = u >> 10;
  const int kb = static_cast<int>(rest % KB), t = static_cast<int>(rest / KB);
  const int n = t * kW8Rows + r;
  const int64_t kw = static_cast<int64_t>(kb) * 16 + pair * 2 + half;  // source word: elements 8kw..8kw+7
  uint32_t out = 0;
  if (n < N) {
    const uint32_t src = (layout_kn ? data[kw * N + n] : data[static_cast<int64_t>(n) * (K / 8) + kw]) ^ 0x88888888u;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t nib = (src >> (order_high ? 28 - 4 * j : 4 * j)) & 15u;
      out |= nib << (4 * (j < 4 ? 2 * j : 2 * (j - 4) + 1));
    }
  }
  tiles[i] = out;
}

// PackedInt4 fp32 scales and int32 zeros (z = zu - 8) -> {scale bits, zu}.
__global__ void w4a8_groups_kernel(const float* __restrict__ scales, const int32_t* __restrict__ zeros, int N,
                                   int G, int64_t total, uint64_t* __restrict__ groups) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int r = static_cast<int>(i & 127);
  const int64_t rest = i >> 7;
  const int g = static_cast<int>(rest % G), t = static_cast<int>(rest / G);
  const int n = t * kW8Rows + r;
  uint64_t v = 0;
  if (n < N) {
    const int64_t src = static_cast<int64_t>(n) * G + g;
    v = static_cast<uint64_t>(__float_as_uint(scales[src])) |
        (static_cast<uint64_t>(static_cast<uint32_t>(zeros[src] + 8)) << 32);
  }
  groups[i] = v;
}

// ----------------------------------------------------------------- host
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn tensor_map_encoder();

size_t w4a8_tiles_bytes(int64_t N, int64_t K) {
  return static_cast<size_t>((N + kW8Rows - 1) / kW8Rows) * (K / 128) * kW8Chunk;
}

size_t w4a8_groups_bytes(int64_t N, int64_t K, int group) {
  return static_cast<size_t>((N + kW8Rows - 1) / kW8Rows) * (K / group) * kW8Rows * 8;
}

size_t w4a8_workspace(int64_t M, int64_t K, int group) {
  const int64_t mp = (M + 15) / 16 * 16 + kW8MaxBT;  // a tile's 16-token slices never read past the end
  return (static_cast<size_t>(mp) * (K / group) * 4 + 255) / 256 * 256;
}

cudaError_t run_w4a8_prepare(const uint32_t* data, int layout_kn, int order_high, const float* scales,
                             const int32_t* zeros, int64_t N, int64_t K, int group, void* tiles, void* groups,
                             cudaStream_t stream) {
  const int64_t tw = static_cast<int64_t>(w4a8_tiles_bytes(N, K) / 4);
  const int64_t gw = static_cast<int64_t>(w4a8_groups_bytes(N, K, group) / 8);
  if (tw == 0) return cudaSuccess;
  w4a8_tiles_kernel<<<static_cast<unsigned>((tw + 255) / 256), 256, 0, stream>>>(
      data, layout_kn, order_high, static_cast<int>(N), static_cast<int>(K), static_cast<int>(K / 128), tw,
      static_cast<uint32_t*>(tiles));
  w4a8_groups_kernel<<<static_cast<unsigned>((gw + 255) / 256), 256, 0, stream>>>(
      scales, zeros, static_cast<int>(N), static_cast<int>(K / group), gw, static_cast<uint64_t*>(groups));
  return cudaGetLastError();
}

template <int BT, int RK, int RS>
static cudaError_t launch_w4a8(const int8_t* a, int64_t lda, const W4A8Params& p, cudaStream_t stream) {
  using L = W8Layout<BT, RK, RS>;
  auto kernel = w4a8_kernel<BT, RK, RS>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  EncodeTiledFn fn = tensor_map_encoder();
  if (fn == nullptr) return cudaErrorNotSupported;
  CUtensorMap ma;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(p.K), static_cast<cuuint64_t>(p.M)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(lda)};
  const cuuint32_t box[2] = {128, static_cast<cuuint32_t>(BT)};
  const cuuint32_t estr[2] = {1, 1};
  if (fn(&ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(a), dims, strides, box, estr,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  kernel<<<p.P, L::kThreads, L::kAlloc, stream>>>(ma, p);
  return cudaGetLastError();
}

cudaError_t run_w4a8(const int8_t* a, int64_t lda, const void* tiles, const void* groups, int group, int64_t M,
                     int64_t N, int64_t K, const float* a_scale, const void* bias, int bias_dtype, int integer,
                     void* out, int64_t ldo, void* workspace, cudaStream_t stream) {
  if (M == 0 || N == 0) return cudaSuccess;
  // Token tile: 16 / 32 for decode sizes, 64 from M = 64 up (MMA N = 64
  // halves the issue cost per token; bit-identical results -- every group is
  // an exact int32 dot -- and at the config-3 shape M=128 102 -> 79 us,
  // M=2048 1153 -> 773 us, though the 64-token drain spills a little).
  const int bt = M <= 16 ? 16 : M < 64 ? 32 : 64;
  W4A8Params p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.group = group;
  p.T = static_cast<int>((N + kW8Rows - 1) / kW8Rows);
  p.KB = static_cast<int>(K / 128);
  p.G = static_cast<int>(K / group);
  p.TM = static_cast<int>((M + bt - 1) / bt);
  const int64_t tiles_total = static_cast<int64_t>(p.T) * p.TM;
  const int sms = device_sm_count();
  p.P = static_cast<int>(tiles_total < sms ? tiles_total : sms);
  p.integer = integer;
  p.groups = static_cast<const uint64_t*>(groups);
  p.tiles = static_cast<const uint8_t*>(tiles);
  p.a_scale = a_scale;
  p.asum = static_cast<const int32_t*>(workspace);
  p.Mp = static_cast<int>((M + 15) / 16 * 16 + kW8MaxBT);
  p.bias = bias;
  p.bias_dtype = bias_dtype;
  p.out = out;
  p.ldo = ldo;
  p.status = status_word_ptr();
  const int64_t na = static_cast<int64_t>(p.Mp) * p.G;
  w4a8_asum_kernel<<<static_cast<unsigned>((na + 255) / 256), 256, 0, stream>>>(
      a, lda, p.M, p.Mp, p.K, group, static_cast<int32_t*>(workspace));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (bt == 64) return launch_w4a8<64, 4, 2>(a, lda, p, stream);
  if (bt == 16) return launch_w4a8<16, 4, 4>(a, lda, p, stream);
  return launch_w4a8<32, 4, 4>(a, lda, p, stream);
}

}  // namespace b2
