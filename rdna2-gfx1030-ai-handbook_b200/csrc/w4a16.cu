// W4A16 weight-only GEMM for sm_100a: y[m,n] = sum_k a[m,k] * w[n,k] (+bias[n]),
// with w[n,k] = round_to_16bit((u[n,k] - zu[n,g]) * s[n,g]), g = k / group.
//
// Replaces int4_linear_a16 / _linear_dot2 of the reference
// (rdna2_ops/int4_weight_gemm_v07.py:540-564, 365-387), which decodes each
// weight as ((q - z).to(fp32) * s).to(fp16) inside the K loop and
// accumulates 16-bit x 16-bit products in fp32.
//
// Weight format ("W4A16 tiles"; b2_w4a16_prepare builds it from PackedInt4):
//   tiles  u32 [T][KB][128][8], T = ceil(N/128) row tiles, KB = K/64: one
//          4 KiB chunk per (row tile, k-block) holding 128 rows x 64 unsigned
//          nibbles u = q + 8.  Inside a word, element j = k % 8 sits at nibble
//          (j >> 1) + 4 * (j & 1), so masking nibbles {i, i + 4} yields
//          elements (2i, 2i + 1) as the two halves of a 32-bit word.
//   groups u32 [T][G][128], G = K / group: low half the scale s, high half
//          the zero point zu (an integer 0..15), both in the activation's
//          16-bit type.  Rows past N are zero.
// Chunks are stored in (tile, k-block) order, so the weights a CTA streams
// form one contiguous byte range, fetched by bulk copies of up to 16 KiB
// (whole DRAM pages) rather than 32-byte pieces of 128 separate rows.
//
// B200 design (both kernels):
//  * swap-AB: the dequantized weight tile is the 128-row A operand of
//    tcgen05.mma kind::f16 and the tokens are its N dimension (BT = 16..256).
//  * persistent, one CTA per SM; warp 0 streams a raw ring (RK k-blocks of
//    words + their group operands by bulk copy, activation tiles by TMA);
//    dequantization is exact sub then one rounded mul per weight, stored
//    straight into the 128B-swizzled K-major layout the MMA reads; loops that
//    issue bulk copies or MMAs run on a whole converged warp with one elected
//    lane issuing.
//  * w4a16_decode_kernel, M <= 32 (HBM-bound): stream-K -- the T*KB
//    (tile, k-block) units are divided evenly over the CTAs.  Three transform
//    groups each own every third k-block, dequantize it into one of two
//    ping-pong slots and issue its MMAs themselves into a per-group TMEM
//    accumulator (no hand-off per k-block).  A tile split across CTAs is
//    finished by the CTA covering its first k-blocks (see its epilogue); the
//    sums run in fixed order, so results are run-to-run deterministic.
//  * w4a16_kernel, M > 32: whole (row tile, token tile) pairs round-robin
//    over the CTAs; XS transform groups of 4*UK warps fill UK-k-block slots,
//    one MMA warp issues, TMEM double-buffers the accumulator so the
//    epilogue of one tile overlaps the next.
#include "b2_common.cuh"
#include "b2_internal.h"

namespace b2 {

constexpr int kW4Rows = 128;         // weight rows per tile (UMMA M)
constexpr int kW4Chunk = 4096;       // bytes of one (tile, k-block) of words
constexpr int kW4GroupBytes = 512;   // bytes of one (tile, group) of operands
// Decode workspace: arrival counters first (one per CTA, fixed capacity so
// that workspaces reused across shapes never put slots over counters), then
// the fp32 partial slots.
constexpr int kW4MaxCtas = 1024;
constexpr size_t kW4CounterBytes = kW4MaxCtas * 4;

struct W4Params {
  int M, N, K;
  int gshift;              // log2(group)
  int T, KB, G, TM;        // row tiles, k-blocks, groups, token tiles
  int P;                   // CTAs in the grid
  int streamk;             // 1: stream-K partial slots, 0: whole tiles
  int64_t U;               // T * KB units (stream-K)
  const uint8_t* tiles;
  const uint8_t* groups;
  const void* bias;
  int bias_dtype;
  void* out;
  int64_t ldo;
  float* partial;          // [T + P - 1][128][BT] fp32 (stream-K)
  int* counters;           // [P] arrivals at the tile finished by each CTA, zero at launch
  int* status;
};

struct W4Seg {
  int tn, tm, kb0, kb1, slot;
};

// First unit of CTA c under the even stream-K split.
__host__ __device__ __forceinline__ int64_t w4_begin(int64_t U, int P, int c) {
  return (static_cast<int64_t>(c) * U) / P;
}
// The CTA whose range holds unit u (inverse of w4_begin).
__host__ __device__ __forceinline__ int w4_owner(int64_t U, int P, int64_t u) {
  return static_cast<int>(((u + 1) * P - 1) / U);
}

__device__ __forceinline__ int64_t w4_first(const W4Params& p) {
  return p.streamk ? w4_begin(p.U, p.P, blockIdx.x) : static_cast<int64_t>(blockIdx.x);
}

// Next segment of this CTA's work; every role walks the same sequence.
__device__ __forceinline__ bool w4_next(const W4Params& p, int64_t& cursor, W4Seg& s) {
  if (p.streamk) {
    const int64_t end = w4_begin(p.U, p.P, blockIdx.x + 1);
    if (cursor >= end) return false;
    const int x = static_cast<int>(cursor / p.KB);
    const int64_t base = static_cast<int64_t>(x) * p.KB;
    const int64_t e = base + p.KB < end ? base + p.KB : end;
    s.tn = x;
    s.tm = 0;
    s.kb0 = static_cast<int>(cursor - base);
    s.kb1 = static_cast<int>(e - base);
    s.slot = x + static_cast<int>(blockIdx.x);
    cursor = e;
    return true;
  }
  if (cursor >= static_cast<int64_t>(p.T) * p.TM) return false;
  const int x = static_cast<int>(cursor);
  s.tn = x / p.TM;
  s.tm = x % p.TM;
  s.kb0 = 0;
  s.kb1 = p.KB;
  s.slot = -1;
  cursor += p.P;
  return true;
}

// One word of 8 interleaved nibbles -> 8 16-bit weights (one 16-byte chunk)
// in K order.  0x4300 | u is bf16 128 + u, 0x6400 | u is fp16 1024 + u; the
// subtraction of 128 + zu (1024 + zu) is exact, the product rounds once.
template <bool BF16>
__device__ __forceinline__ uint4 dequant_word(uint32_t w, uint32_t zz, uint32_t ss) {
  constexpr uint32_t kBias = BF16 ? 0x43004300u : 0x64006400u;
  uint32_t r[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t t = ((w >> (4 * i)) & 0x000F000Fu) | kBias;  // elements (2i, 2i+1)
    if constexpr (BF16) {
      const __nv_bfloat162 d = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&t),
                                       *reinterpret_cast<const __nv_bfloat162*>(&zz));
      const __nv_bfloat162 v = __hmul2(d, *reinterpret_cast<const __nv_bfloat162*>(&ss));
      r[i] = *reinterpret_cast<const uint32_t*>(&v);
    } else {
      const __half2 d = __hsub2(*reinterpret_cast<const __half2*>(&t), *reinterpret_cast<const __half2*>(&zz));
      const __half2 v = __hmul2(d, *reinterpret_cast<const __half2*>(&ss));
      r[i] = *reinterpret_cast<const uint32_t*>(&v);
    }
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

// Group operand word {s, zu} -> {128+zu, 128+zu} (bf16) or {1024+zu, ...}
// (fp16), and {s, s}.
template <bool BF16>
__device__ __forceinline__ void group_operands(uint32_t sz, uint32_t& zz, uint32_t& ss) {
  ss = __byte_perm(sz, 0u, 0x1010);
  const uint32_t z2 = __byte_perm(sz, 0u, 0x3232);
  constexpr uint32_t kBias = BF16 ? 0x43004300u : 0x64006400u;
  if constexpr (BF16) {
    const __nv_bfloat162 v = __hadd2(*reinterpret_cast<const __nv_bfloat162*>(&z2),
                                     *reinterpret_cast<const __nv_bfloat162*>(&kBias));
    zz = *reinterpret_cast<const uint32_t*>(&v);
  } else {
    const __half2 v = __hadd2(*reinterpret_cast<const __half2*>(&z2), *reinterpret_cast<const __half2*>(&kBias));
    zz = *reinterpret_cast<const uint32_t*>(&v);
  }
}

template <int BT, int RK, int RS, int XS, int UK>
struct W4Layout {
  static constexpr int kXfBlock = kW4Rows * 128;       // 128 rows x 64 16-bit, SW128
  static constexpr int kXf = UK * kXfBlock;            // one slot: UK k-blocks
  static constexpr int kAct = BT * 128;                // BT rows x 64 16-bit, SW128
  static constexpr int kWords = RK * kW4Chunk;
  static constexpr int kGrp = 2 * RK * kW4GroupBytes;  // <= 2*RK groups per stage (group >= 32)
  static constexpr int kOffXf = 0;
  static constexpr int kOffAct = kOffXf + XS * kXf;
  static constexpr int kOffWords = kOffAct + RS * RK * kAct;
  static constexpr int kOffGrp = kOffWords + RS * kWords;
  static constexpr int kOffBar = kOffGrp + RS * kGrp;
  static constexpr int kNumBars = 2 * RS + 2 * XS + 5;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  // misc: [0] TMEM base, [4] abort flag
  static constexpr int kAlloc = kOffMisc + 16 + 1024;  // + alignment slack
  static constexpr uint32_t kTmemCols = 2 * BT < 32 ? 32 : 2 * BT;
  static constexpr int kGroupWarps = 4 * UK;           // one thread per (row, k-block of the unit)
  static constexpr int kXfWarps = XS * kGroupWarps;
  static_assert(kAlloc <= 232448, "shared memory budget");
  static_assert(kAct % 1024 == 0, "SW128 tiles need 1 KiB alignment");
  static_assert(RK % UK == 0, "a raw stage holds whole units");
};

template <int BT, int RK, int RS, int XS, int UK>
constexpr int w4_threads() {
  return 64 + 32 * W4Layout<BT, RK, RS, XS, UK>::kXfWarps + 128;
}

template <bool BF16, int BT, int RK, int RS, int XS, int UK>
__global__ void __launch_bounds__(w4_threads<BT, RK, RS, XS, UK>(), 1)
    w4a16_kernel(const __grid_constant__ CUtensorMap tma_a, const W4Params p) {
  using L = W4Layout<BT, RK, RS, XS, UK>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint64_t* full_raw = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* raw_empty = full_raw + RS;
  uint64_t* full_xf = raw_empty + RS;
  uint64_t* xf_empty = full_xf + XS;
  uint64_t* acc_full = xf_empty + XS;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kEpiWarp0 = 2 + L::kXfWarps;

  if (threadIdx.x == 0) {
    for (int s = 0; s < RS; ++s) {
      mbar_init(&full_raw[s], 1);
      mbar_init(&raw_empty[s], L::kXfWarps + 1);  // every transform warp + the MMA commit
    }
    for (int s = 0; s < XS; ++s) {
      mbar_init(&full_xf[s], L::kGroupWarps);  // the slot's transform group
      mbar_init(&xf_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tma_a);
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---- producer: words + group operands (bulk) and activation tiles (TMA).
    // The whole warp runs the loop and one elected lane issues: a loop run
    // by a single lane of a diverged warp pays a large per-iteration cost.
    int rs = 0;
    uint32_t rph = 0, live = 0, live_par = 0;
    bool ok = true;
    int64_t cur = w4_first(p);
    W4Seg s;
    while (ok && w4_next(p, cur, s)) {
      for (int kb = s.kb0; kb < s.kb1; kb += RK) {
        const int n = s.kb1 - kb < RK ? s.kb1 - kb : RK;
        const int g_lo = (kb * 64) >> p.gshift, g_hi = ((kb + n) * 64 - 1) >> p.gshift;
        const int ng = g_hi - g_lo + 1;
        ok = __all_sync(0xffffffffu, mbar_wait(&raw_empty[rs], rph ^ 1u, abort_flag, kSiteProducer, p.status));
        if (!ok) break;
        if (elect_one()) {
          mbar_arrive_expect_tx(&full_raw[rs], static_cast<uint32_t>(n * (kW4Chunk + L::kAct) + ng * kW4GroupBytes));
          bulk_load(smem + L::kOffWords + rs * L::kWords,
                    p.tiles + (static_cast<int64_t>(s.tn) * p.KB + kb) * kW4Chunk, n * kW4Chunk, &full_raw[rs]);
          bulk_load(smem + L::kOffGrp + rs * L::kGrp,
                    p.groups + (static_cast<int64_t>(s.tn) * p.G + g_lo) * kW4GroupBytes, ng * kW4GroupBytes,
                    &full_raw[rs]);
          for (int j = 0; j < n; ++j)
            tma_load_2d(&tma_a, &full_raw[rs], smem + L::kOffAct + (rs * RK + j) * L::kAct, (kb + j) * 64, s.tm * BT);
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
    for (int i = 0; i < RS && ok; ++i) {  // tail: every stage released
      ok = __all_sync(0xffffffffu, mbar_wait(&raw_empty[rs], rph ^ 1u, abort_flag, kSiteProducer, p.status));
      if (++rs == RS) {
        rs = 0;
        rph ^= 1u;
      }
    }
    if (!ok && lane == 0) {  // copies issued before an abort still land here: let them finish
      const uint64_t t0 = globaltimer();
      for (int i = 0; i < RS; ++i)
        if ((live >> i) & 1u)
          while (!mbar_try_wait(&full_raw[i], (live_par >> i) & 1u) && globaltimer() - t0 < kWaitLimitNs) {
          }
    }
  } else if (warp == 1) {
    // ---- MMA issuer: one wait and one commit per unit of UK k-blocks.  The
    // whole warp runs the loop, one elected lane issues (the same lane every
    // time, so its commits cover its own MMAs).
    constexpr uint32_t idesc = (1u << 4) | (BF16 ? (1u << 7) | (1u << 10) : 0u) |
                               (static_cast<uint32_t>(BT >> 3) << 17) |
                               (static_cast<uint32_t>(kW4Rows >> 4) << 24);
    // Descriptors are computed once; a tile's start address sits in the low
    // 14 bits (address >> 4), so stepping slots and K slices is an add.
    const uint64_t a_desc0 = sw128_desc(smem_u32(smem + L::kOffXf));
    const uint64_t b_desc0 = sw128_desc(smem_u32(smem + L::kOffAct));
    int rs = 0, xs = 0, seg_i = 0;
    uint32_t xph = 0;
    bool ok = true;
    int64_t cur = w4_first(p);
    W4Seg s;
    while (ok && w4_next(p, cur, s)) {
      const int b = seg_i & 1;
      ok = __all_sync(0xffffffffu,
                      mbar_wait(&acc_empty[b], ((seg_i >> 1) & 1) ^ 1u, abort_flag, kSiteMmaTmem, p.status));
      if (!ok) break;
      tc_fence_after();
      const uint32_t d = tmem_base + static_cast<uint32_t>(b * BT);
      uint32_t acc = 0;
      for (int kb = s.kb0; kb < s.kb1 && ok; kb += RK) {
        const int n = s.kb1 - kb < RK ? s.kb1 - kb : RK;
        const uint64_t b_stage = b_desc0 + static_cast<uint32_t>((rs * RK * L::kAct) >> 4);
        for (int u0 = 0; u0 < n; u0 += UK) {
          const int nk = n - u0 < UK ? n - u0 : UK;
          ok = __all_sync(0xffffffffu, mbar_wait(&full_xf[xs], xph, abort_flag, kSiteMma, p.status));
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            const uint64_t ad0 = a_desc0 + static_cast<uint32_t>((xs * L::kXf) >> 4);
            const uint64_t bd0 = b_stage + static_cast<uint32_t>((u0 * L::kAct) >> 4);
#pragma unroll
            for (int h = 0; h < UK; ++h) {
              if (h < nk) {
                const uint64_t ad = ad0 + static_cast<uint32_t>((h * L::kXfBlock) >> 4);
                const uint64_t bd = bd0 + static_cast<uint32_t>((h * L::kAct) >> 4);
                umma<kKindBF16>(d, ad, bd, idesc, h == 0 ? acc : 1u);
                umma<kKindBF16>(d, ad + 2, bd + 2, idesc, 1u);
                umma<kKindBF16>(d, ad + 4, bd + 4, idesc, 1u);
                umma<kKindBF16>(d, ad + 6, bd + 6, idesc, 1u);
              }
            }
            umma_commit(&xf_empty[xs]);
          }
          __syncwarp();
          acc = 1;
          if (++xs == XS) {
            xs = 0;
            xph ^= 1u;
          }
        }
        if (!ok) break;
        if (elect_one()) umma_commit(&raw_empty[rs]);
        __syncwarp();
        if (++rs == RS) rs = 0;
      }
      if (!ok) break;
      if (elect_one()) umma_commit(&acc_full[b]);
      __syncwarp();
      ++seg_i;
    }
    // Every MMA issued above completes before TMEM is released.
    if (elect_one()) {
      umma_commit(drain);
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < kWaitLimitNs) {
      }
    }
    __syncwarp();
  } else if (warp < kEpiWarp0) {
    // ---- transform: XS groups of 4*UK warps.  Group gi dequantizes units
    // i = gi, gi + XS, ... of this CTA's unit sequence into slot gi; thread
    // (sub, r) handles k-block `sub` of the unit for weight row r (64
    // elements).  XS units are in flight at once.
    const int t = threadIdx.x - 64;
    const int gi = t / (128 * UK), sub = (t / 128) % UK, r = t & 127;
    // Natural half order: each 16-byte store of a quarter-warp (8 rows)
    // lands on 8 distinct chunk columns of the 128B swizzle (conflict-free);
    // the two 16-byte loads of the packed words are 2-way conflicted instead,
    // the cheaper side of the trade (2 loads against 8 stores per k-block).
    constexpr int ha = 0;
    // Row r of k-block `sub` of slot gi, 128B swizzle: 16-byte chunk c lives
    // at chunk c ^ (r & 7).
    const uint32_t xrow =
        (smem_u32(smem + L::kOffXf + gi * L::kXf + sub * L::kXfBlock) + r * 128) | ((r & 7) << 4);
    const uint32_t xa = xrow ^ ((4 * ha) << 4), xb = xrow ^ ((4 * (ha ^ 1)) << 4);
    int rs = 0, i = 0;
    uint32_t rph = 0, use = 0;
    bool ok = true;
    int64_t cur = w4_first(p);
    W4Seg s;
    while (ok && w4_next(p, cur, s)) {
      for (int kb = s.kb0; kb < s.kb1; kb += RK) {
        const int n = s.kb1 - kb < RK ? s.kb1 - kb : RK;
        const int g_lo = (kb * 64) >> p.gshift;
        ok = __all_sync(0xffffffffu, mbar_wait(&full_raw[rs], rph, abort_flag, kSiteTransform, p.status));
        if (!ok) break;
        const uint32_t words = smem_u32(smem + L::kOffWords + rs * L::kWords) + r * 32;
        const uint32_t grp = smem_u32(smem + L::kOffGrp + rs * L::kGrp) + r * 4;
        for (int u0 = 0; u0 < n; u0 += UK, ++i) {
          if (i % XS != gi) continue;
          ok = __all_sync(0xffffffffu, mbar_wait(&xf_empty[gi], use ^ 1u, abort_flag, kSiteTransform, p.status));
          if (!ok) break;
          const int j = u0 + sub;  // k-block of this stage handled by this thread
          if (j < n) {
            const uint4 wa = lds_v4(words + j * kW4Chunk + ha * 16);
            const uint4 wb = lds_v4(words + j * kW4Chunk + (ha ^ 1) * 16);
            const int ga = (((kb + j) * 64 + ha * 32) >> p.gshift) - g_lo;
            const int gb = (((kb + j) * 64 + (ha ^ 1) * 32) >> p.gshift) - g_lo;
            uint32_t za, sa, zb, sb;
            group_operands<BF16>(lds_u32(grp + ga * kW4Rows * 4), za, sa);
            group_operands<BF16>(lds_u32(grp + gb * kW4Rows * 4), zb, sb);
            sts_v4(xa ^ (0 << 4), dequant_word<BF16>(wa.x, za, sa));
            sts_v4(xa ^ (1 << 4), dequant_word<BF16>(wa.y, za, sa));
            sts_v4(xa ^ (2 << 4), dequant_word<BF16>(wa.z, za, sa));
            sts_v4(xa ^ (3 << 4), dequant_word<BF16>(wa.w, za, sa));
            sts_v4(xb ^ (0 << 4), dequant_word<BF16>(wb.x, zb, sb));
            sts_v4(xb ^ (1 << 4), dequant_word<BF16>(wb.y, zb, sb));
            sts_v4(xb ^ (2 << 4), dequant_word<BF16>(wb.z, zb, sb));
            sts_v4(xb ^ (3 << 4), dequant_word<BF16>(wb.w, zb, sb));
            fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core
          }
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
    // ---- epilogue: TMEM lane = weight row, column = token
    const int quarter = warp & 3;
    const int rt = quarter * 32 + lane;
    int seg_i = 0;
    bool ok = true;
    int64_t cur = w4_first(p);
    W4Seg s;
    while (ok && w4_next(p, cur, s)) {
      const int b = seg_i & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[b], (seg_i >> 1) & 1, abort_flag, kSiteEpilogue, p.status));
      if (!ok) break;
      tc_fence_after();
      const int n = s.tn * kW4Rows + rt;
      const int m0 = s.tm * BT;
      const int mc = p.M - m0 < BT ? p.M - m0 : BT;
      float bias = 0.0f;
      if (p.bias != nullptr && n < p.N) bias = load_as_float(p.bias, p.bias_dtype, n);
#pragma unroll 1
      for (int c0 = 0; c0 < mc; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(b * BT + c0), v);
        tmem_ld_wait16(v);
        if (n < p.N) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (c0 + j < mc) {
              const float y = __fadd_rn(__uint_as_float(v[j]), bias);
              uint16_t* o = static_cast<uint16_t*>(p.out) + static_cast<int64_t>(m0 + c0 + j) * p.ldo + n;
              *o = BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(y)) : __half_as_ushort(__float2half_rn(y));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
      ++seg_i;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// Bounded wait until *ctr >= target (acquire: the publishers' slot stores
// are visible afterwards).  False after kWaitLimitNs or an abort.
__device__ __forceinline__ bool wait_count(const int* ctr, int target, volatile int* abort_flag, int* status) {
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 0;; ++it) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
    if (v >= target) return true;
    if ((it & 15u) == 15u) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > kWaitLimitNs) {
        *abort_flag = 1;
        if (status != nullptr) atomicCAS(status, 0, 0x100 | kSiteFixup);
        return false;
      }
    }
    __nanosleep(64);
  }
}

// ------------------------------------------------------------------ decode
// Decode kernel (M <= 32, stream-K).  NG groups, each of 4 transform warps
// and its own MMA warp: group g owns the k-blocks i = g, g + NG, ... of this
// CTA's k-block sequence, dequantizes them into its two ping-pong slots and
// accumulates them into its own TMEM accumulator, so a group's MMA warp
// handles only every NG-th k-block and no transform warp ever waits on MMA
// issue.  The epilogue sums a segment's NG accumulators in group order
// (deterministic).
template <int BT, int RK, int RS, int NG>
struct W4DecLayout {
  static constexpr int kXf = kW4Rows * 128;            // one k-block slot, SW128
  static constexpr int kAct = BT * 128;
  static constexpr int kWords = RK * kW4Chunk;
  static constexpr int kGrp = 2 * RK * kW4GroupBytes;
  static constexpr int kOffXf = 0;                     // [NG][2] slots
  static constexpr int kOffAct = kOffXf + NG * 2 * kXf;
  static constexpr int kOffWords = kOffAct + RS * RK * kAct;
  static constexpr int kOffGrp = kOffWords + RS * kWords;
  static constexpr int kOffBar = kOffGrp + RS * kGrp;
  static constexpr int kNumBars = 2 * RS + 4 * NG + 5;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  // misc: [0] TMEM base, [4] abort flag
  static constexpr int kAlloc = kOffMisc + 16 + 1024;
  static constexpr uint32_t kCols = 2 * NG * BT;       // [buffer][group] accumulators
  static constexpr uint32_t kTmemCols = kCols <= 32 ? 32 : kCols <= 64 ? 64 : kCols <= 128 ? 128 : kCols <= 256 ? 256 : 512;
  // warps: producer, NG MMA warps (the first also owns TMEM), NG groups of 4
  // transform warps, 4 epilogue warps
  static constexpr int kMmaWarp0 = 1;
  static constexpr int kXfWarp0 = 1 + NG;
  static constexpr int kEpiWarp0 = kXfWarp0 + 4 * NG;
  static constexpr int kThreads = 32 * (kEpiWarp0 + 4);
  static_assert(kAlloc <= 232448, "shared memory budget");
  static_assert(kCols <= 512, "TMEM budget");
  static_assert(BT <= 32, "decode token tiles");
};

template <bool BF16, int BT, int RK, int RS, int NG>
__global__ void __launch_bounds__(W4DecLayout<BT, RK, RS, NG>::kThreads, 1)
    w4a16_decode_kernel(const __grid_constant__ CUtensorMap tma_a, const W4Params p) {
  using L = W4DecLayout<BT, RK, RS, NG>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint64_t* full_raw = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* raw_empty = full_raw + RS;
  uint64_t* slot_full = raw_empty + RS;    // [NG][2]
  uint64_t* slot_empty = slot_full + 2 * NG;  // [NG][2]
  uint64_t* acc_full = slot_empty + 2 * NG;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kEpiWarp0 = L::kEpiWarp0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < RS; ++s) {
      mbar_init(&full_raw[s], 1);
      mbar_init(&raw_empty[s], 4 * NG + NG);  // every transform warp + each MMA warp's commit
    }
    for (int s = 0; s < 2 * NG; ++s) {
      mbar_init(&slot_full[s], 4);   // the group's transform warps
      mbar_init(&slot_empty[s], 1);  // the group's MMA commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], NG);  // one commit per MMA warp
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(drain, NG);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tma_a);
  if (warp == L::kMmaWarp0) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---- producer (whole warp loops, one elected lane issues)
    int rs = 0;
    uint32_t rph = 0, live = 0, live_par = 0;
    bool ok = true;
    int64_t cur = w4_first(p);
    W4Seg s;
    while (ok && w4_next(p, cur, s)) {
      for (int kb = s.kb0; kb < s.kb1; kb += RK) {
        const int n = s.kb1 - kb < RK ? s.kb1 - kb : RK;
        const int g_lo = (kb * 64) >> p.gshift, g_hi = ((kb + n) * 64 - 1) >> p.gshift;
        const int ng = g_hi - g_lo + 1;
        ok = __all_sync(0xffffffffu, mbar_wait(&raw_empty[rs], rph ^ 1u, abort_flag, kSiteProducer, p.status));
        if (!ok) break;
        if (elect_one()) {
          mbar_arrive_expect_tx(&full_raw[rs], static_cast<uint32_t>(n * (kW4Chunk + L::kAct) + ng * kW4GroupBytes));
          bulk_load(smem + L::kOffWords + rs * L::kWords,
                    p.tiles + (static_cast<int64_t>(s.tn) * p.KB + kb) * kW4Chunk, n * kW4Chunk, &full_raw[rs]);
          bulk_load(smem + L::kOffGrp + rs * L::kGrp,
                    p.groups + (static_cast<int64_t>(s.tn) * p.G + g_lo) * kW4GroupBytes, ng * kW4GroupBytes,
                    &full_raw[rs]);
          for (int j = 0; j < n; ++j)
            tma_load_2d(&tma_a, &full_raw[rs], smem + L::kOffAct + (rs * RK + j) * L::kAct, (kb + j) * 64, 0);
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
  } else if (warp < L::kXfWarp0) {
    // ---- MMA warp of group g: the k-blocks i = g, g + NG, ... of this CTA's
    // sequence, into the group's own accumulator.  Whole warp loops, one
    // elected lane (always the same) issues and commits.
    const int g = warp - L::kMmaWarp0;
    constexpr uint32_t idesc = (1u << 4) | (BF16 ? (1u << 7) | (1u << 10) : 0u) |
                               (static_cast<uint32_t>(BT >> 3) << 17) |
                               (static_cast<uint32_t>(kW4Rows >> 4) << 24);
    const uint64_t a_desc0 = sw128_desc(smem_u32(smem + L::kOffXf + 2 * g * L::kXf));
    const uint64_t b_desc0 = sw128_desc(smem_u32(smem + L::kOffAct));
    int rs = 0, i = 0, jg = 0, seg_i = 0;
    bool ok = true;
    int64_t cur = w4_first(p);
    W4Seg s;
    while (ok && w4_next(p, cur, s)) {
      const int b = seg_i & 1;
      const uint32_t d = tmem_base + static_cast<uint32_t>((b * NG + g) * BT);
      ok = __all_sync(0xffffffffu,
                      mbar_wait(&acc_empty[b], ((seg_i >> 1) & 1) ^ 1u, abort_flag, kSiteMmaTmem, p.status));
      if (!ok) break;
      tc_fence_after();
      uint32_t acc = 0;
      for (int kb = s.kb0; kb < s.kb1 && ok; kb += RK) {
        const int n = s.kb1 - kb < RK ? s.kb1 - kb : RK;
        for (int j = 0; j < n; ++j, ++i) {
          if (i % NG != g) continue;
          const int sl = jg & 1;
          ok = __all_sync(0xffffffffu, mbar_wait(&slot_full[2 * g + sl], (jg >> 1) & 1, abort_flag, kSiteMma, p.status));
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            const uint64_t ad = a_desc0 + static_cast<uint32_t>((sl * L::kXf) >> 4);
            const uint64_t bd = b_desc0 + static_cast<uint32_t>(((rs * RK + j) * L::kAct) >> 4);
            umma<kKindBF16>(d, ad, bd, idesc, acc);
            umma<kKindBF16>(d, ad + 2, bd + 2, idesc, 1u);
            umma<kKindBF16>(d, ad + 4, bd + 4, idesc, 1u);
            umma<kKindBF16>(d, ad + 6, bd + 6, idesc, 1u);
            umma_commit(&slot_empty[2 * g + sl]);
          }
          __syncwarp();
          acc = 1;
          ++jg;
        }
        if (!ok) break;
        // the stage's activation tiles are free once this warp's MMAs are done
        if (elect_one()) umma_commit(&raw_empty[rs]);
        __syncwarp();
        if (++rs == RS) rs = 0;
      }
      if (!ok) break;
      if (elect_one()) umma_commit(&acc_full[b]);
      __syncwarp();
      ++seg_i;
    }
    // Before TMEM is released: every MMA of every group complete.
    if (elect_one()) umma_commit(drain);
    __syncwarp();
    if (g == 0 && lane == 0) {
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < kWaitLimitNs) {
      }
    }
    __syncwarp();
  } else if (warp < kEpiWarp0) {
    // ---- transform, group g of 4 warps; thread = weight row r.  Each warp
    // runs on its own (no group barrier): it arrives on the slot's full
    // barrier after its rows are written.
    const int t = threadIdx.x - 32 * L::kXfWarp0;
    const int g = t >> 7, r = t & 127;
    constexpr int ha = 0;  // natural half order (conflict-free 16-byte stores)
    // Slot 1 sits kXf bytes after slot 0: its addresses are slot 0's + kXf.
    const uint32_t base0 = smem_u32(smem + L::kOffXf + 2 * g * L::kXf);
    const uint32_t xrow0 = (base0 + r * 128) | ((r & 7) << 4);
    const uint32_t xa0 = xrow0 ^ ((4 * ha) << 4), xb0 = xrow0 ^ ((4 * (ha ^ 1)) << 4);
    int rs = 0, i = 0, jg = 0;
    uint32_t rph = 0;
    bool ok = true;
    int64_t cur = w4_first(p);
    W4Seg s;
    while (ok && w4_next(p, cur, s)) {
      for (int kb = s.kb0; kb < s.kb1; kb += RK) {
        const int n = s.kb1 - kb < RK ? s.kb1 - kb : RK;
        const int g_lo = (kb * 64) >> p.gshift;
        ok = __all_sync(0xffffffffu, mbar_wait(&full_raw[rs], rph, abort_flag, kSiteTransform, p.status));
        if (!ok) break;
        const uint32_t words = smem_u32(smem + L::kOffWords + rs * L::kWords) + r * 32;
        const uint32_t grp = smem_u32(smem + L::kOffGrp + rs * L::kGrp) + r * 4;
        for (int j = 0; j < n; ++j, ++i) {
          if (i % NG != g) continue;
          const int sl = jg & 1;
          const uint32_t xa = xa0 + sl * L::kXf, xb = xb0 + sl * L::kXf;
          ok = __all_sync(0xffffffffu, mbar_wait(&slot_empty[2 * g + sl], ((jg >> 1) & 1) ^ 1u, abort_flag,
                                                 kSiteTransform, p.status));
          if (!ok) break;
          const uint4 wa = lds_v4(words + j * kW4Chunk + ha * 16);
          const uint4 wb = lds_v4(words + j * kW4Chunk + (ha ^ 1) * 16);
          const int ga = (((kb + j) * 64 + ha * 32) >> p.gshift) - g_lo;
          const int gb = (((kb + j) * 64 + (ha ^ 1) * 32) >> p.gshift) - g_lo;
          uint32_t za, sa, zb, sb;
          group_operands<BF16>(lds_u32(grp + ga * kW4Rows * 4), za, sa);
          group_operands<BF16>(lds_u32(grp + gb * kW4Rows * 4), zb, sb);
          sts_v4(xa ^ (0 << 4), dequant_word<BF16>(wa.x, za, sa));
          sts_v4(xa ^ (1 << 4), dequant_word<BF16>(wa.y, za, sa));
          sts_v4(xa ^ (2 << 4), dequant_word<BF16>(wa.z, za, sa));
          sts_v4(xa ^ (3 << 4), dequant_word<BF16>(wa.w, za, sa));
          sts_v4(xb ^ (0 << 4), dequant_word<BF16>(wb.x, zb, sb));
          sts_v4(xb ^ (1 << 4), dequant_word<BF16>(wb.y, zb, sb));
          sts_v4(xb ^ (2 << 4), dequant_word<BF16>(wb.z, zb, sb));
          sts_v4(xb ^ (3 << 4), dequant_word<BF16>(wb.w, zb, sb));
          fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core
          __syncwarp();
          if (lane == 0) mbar_arrive(&slot_full[2 * g + sl]);
          ++jg;
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[rs]);  // this warp's reads of the stage are over
        if (++rs == RS) {
          rs = 0;
          rph ^= 1u;
        }
      }
    }
  } else {
    // ---- epilogue: TMEM lane = weight row, column = token; sums the NG
    // group accumulators of a segment in group order.  A row tile split
    // across CTAs c_lo..c_hi is finished by c_lo, which covers the tile's
    // first k-blocks at the end of its range; the other CTAs cover it at the
    // start of theirs, publish fp32 slots and bump the tile's arrival
    // counter.  c_lo keeps its own sums in registers, waits (bounded) for the
    // count, adds the slots in CTA order, writes the output and resets the
    // counter to zero for the next call.  Waits only ever point at CTAs of
    // higher index, which finish their part first.
    const int quarter = warp & 3;
    const int rt = quarter * 32 + lane;
    const int e0 = 32 * kEpiWarp0;
    const int me = static_cast<int>(blockIdx.x);
    int seg_i = 0, i0 = 0;
    bool ok = true;
    int64_t cur = w4_first(p);
    W4Seg s;
    while (ok && w4_next(p, cur, s)) {
      const int b = seg_i & 1;
      const int len = s.kb1 - s.kb0;
      ok = bar_and(1, 128, mbar_wait(&acc_full[b], (seg_i >> 1) & 1, abort_flag, kSiteEpilogue, p.status));
      if (!ok) break;
      tc_fence_after();
      const int n = s.tn * kW4Rows + rt;
      const int mc = p.M < BT ? p.M : BT;
      const int64_t u0 = static_cast<int64_t>(s.tn) * p.KB;
      const int c_lo = w4_owner(p.U, p.P, u0), c_hi = w4_owner(p.U, p.P, u0 + p.KB - 1);
      const bool finisher = me == c_lo;
      float y[BT];
#pragma unroll
      for (int j = 0; j < BT; ++j) y[j] = 0.0f;
#pragma unroll
      for (int c0 = 0; c0 < BT; c0 += 16) {
        if (c0 < mc) {
#pragma unroll
          for (int gg = 0; gg < NG; ++gg) {
            // group gg holds k-blocks of this segment iff one is = gg mod NG
            if (len >= NG || (((gg - i0) % NG + NG) % NG) < len) {
              uint32_t v[16];
              tmem_ld16(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                            static_cast<uint32_t>((b * NG + gg) * BT + c0),
                        v);
              tmem_ld_wait16(v);
#pragma unroll
              for (int j = 0; j < 16; ++j) y[c0 + j] = __fadd_rn(y[c0 + j], __uint_as_float(v[j]));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);  // TMEM buffer free for the groups
      if (!finisher) {
        // Publish this CTA's share of the tile (token columns past M are 0).
        float* prow = p.partial + (static_cast<int64_t>(s.slot) * kW4Rows + rt) * BT;
#pragma unroll
        for (int q = 0; q < BT / 4; ++q)
          *reinterpret_cast<float4*>(prow + 4 * q) = make_float4(y[4 * q], y[4 * q + 1], y[4 * q + 2], y[4 * q + 3]);
        __threadfence();
        named_bar_sync(1, 128);
        if (static_cast<int>(threadIdx.x) == e0) atomicAdd(&p.counters[c_lo], 1);
      } else {
        if (c_hi > c_lo) {
          bool arrived = true;
          if (static_cast<int>(threadIdx.x) == e0)
            arrived = wait_count(&p.counters[me], c_hi - c_lo, abort_flag, p.status);
          ok = bar_and(1, 128, arrived);
          if (!ok) break;
          __threadfence();
          for (int c = c_lo + 1; c <= c_hi; ++c) {
            const float4* src =
                reinterpret_cast<const float4*>(p.partial + (static_cast<int64_t>(s.tn + c) * kW4Rows + rt) * BT);
#pragma unroll
            for (int q = 0; q < BT / 4; ++q) {
              const float4 v = __ldcg(src + q);
              y[4 * q] = __fadd_rn(y[4 * q], v.x);
              y[4 * q + 1] = __fadd_rn(y[4 * q + 1], v.y);
              y[4 * q + 2] = __fadd_rn(y[4 * q + 2], v.z);
              y[4 * q + 3] = __fadd_rn(y[4 * q + 3], v.w);
            }
          }
          if (static_cast<int>(threadIdx.x) == e0) p.counters[me] = 0;
        }
        if (n < p.N) {
          const float bias = p.bias != nullptr ? load_as_float(p.bias, p.bias_dtype, n) : 0.0f;
#pragma unroll
          for (int j = 0; j < BT; ++j) {
            if (j < mc) {
              const float o32 = __fadd_rn(y[j], bias);
              uint16_t* o = static_cast<uint16_t*>(p.out) + static_cast<int64_t>(j) * p.ldo + n;
              *o = BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(o32)) : __half_as_ushort(__float2half_rn(o32));
            }
          }
        }
      }
      i0 += len;
      ++seg_i;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == L::kMmaWarp0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

template <int BT, int RK, int RS, int NG, int SA>
struct W4TmLayout {
  static constexpr int kAct = BT * 128;
  static constexpr int kWords = RK * kW4Chunk;
  static constexpr int kGrp = 2 * RK * kW4GroupBytes;
  static constexpr int kOffAct = 0;
  static constexpr int kOffWords = kOffAct + RS * RK * kAct;
  static constexpr int kOffGrp = kOffWords + RS * kWords;
  static constexpr int kOffBar = kOffGrp + RS * kGrp;
  static constexpr int kNumBars = 2 * RS + 2 * NG * SA + 5;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  // misc: [0] TMEM base, [4] abort flag
  static constexpr int kAlloc = kOffMisc + 16 + 1024;
  static constexpr uint32_t kCols = 2 * NG * BT;       // [buffer][group] accumulators
  static constexpr uint32_t kSlot0 = (kCols + 31) / 32 * 32;  // [group][SA] dequantized k-blocks, 32 columns each
  static constexpr uint32_t kTmemCols = 512;
  static_assert(kSlot0 + NG * SA * 32 <= kTmemCols, "TMEM budget");
  // warps: producer, NG MMA warps (the first also owns TMEM), NG groups of 4
  // transform warps, 4 epilogue warps
  static constexpr int kMmaWarp0 = 1;
  static constexpr int kXfWarp0 = 1 + NG;
  static constexpr int kEpiWarp0 = kXfWarp0 + 4 * NG;
  static constexpr int kThreads = 32 * (kEpiWarp0 + 4);
  static_assert(kAlloc <= 232448, "shared memory budget");
  static_assert(BT <= 32, "decode token tiles");
  static_assert(kXfWarp0 % 4 == 0, "transform warp q of a group must own TMEM lanes 32q..32q+31");
};

template <bool BF16, int BT, int RK, int RS, int NG, int SA>
__global__ void __launch_bounds__(W4TmLayout<BT, RK, RS, NG, SA>::kThreads, 1)
    w4a16_decode_tm_kernel(const __grid_constant__ CUtensorMap tma_a, const W4Params p) {
  using L = W4TmLayout<BT, RK, RS, NG, SA>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint64_t* full_raw = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* raw_empty = full_raw + RS;
  uint64_t* slot_full = raw_empty + RS;        // [NG][SA]
  uint64_t* slot_empty = slot_full + NG * SA;  // [NG][SA]
  uint64_t* acc_full = slot_empty + NG * SA;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kEpiWarp0 = L::kEpiWarp0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < RS; ++s) {
      mbar_init(&full_raw[s], 1);
      mbar_init(&raw_empty[s], 4 * NG + NG);  // every transform warp + each MMA warp's commit
    }
    for (int s = 0; s < NG * SA; ++s) {
      mbar_init(&slot_full[s], 4);   // the group's transform warps
      mbar_init(&slot_empty[s], 1);  // the group's MMA commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], NG);  // one commit per MMA warp
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(drain, NG);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tma_a);
  if (warp == L::kMmaWarp0) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---- producer (whole warp loops, one elected lane issues)
    int rs = 0;
    uint32_t rph = 0, live = 0, live_par = 0;
    bool ok = true;
    int64_t cur = w4_first(p);
    W4Seg s;
    while (ok && w4_next(p, cur, s)) {
      for (int kb = s.kb0; kb < s.kb1; kb += RK) {
        const int n = s.kb1 - kb < RK ? s.kb1 - kb : RK;
        const int g_lo = (kb * 64) >> p.gshift, g_hi = ((kb + n) * 64 - 1) >> p.gshift;
        const int ng = g_hi - g_lo + 1;
        ok = __all_sync(0xffffffffu, mbar_wait(&raw_empty[rs], rph ^ 1u, abort_flag, kSiteProducer, p.status));
        if (!ok) break;
        if (elect_one()) {
          mbar_arrive_expect_tx(&full_raw[rs], static_cast<uint32_t>(n * (kW4Chunk + L::kAct) + ng * kW4GroupBytes));
          bulk_load(smem + L::kOffWords + rs * L::kWords,
                    p.tiles + (static_cast<int64_t>(s.tn) * p.KB + kb) * kW4Chunk, n * kW4Chunk, &full_raw[rs]);
          bulk_load(smem + L::kOffGrp + rs * L::kGrp,
                    p.groups + (static_cast<int64_t>(s.tn) * p.G + g_lo) * kW4GroupBytes, ng * kW4GroupBytes,
                    &full_raw[rs]);
          for (int j = 0; j < n; ++j)
            tma_load_2d(&tma_a, &full_raw[rs], smem + L::kOffAct + (rs * RK + j) * L::kAct, (kb + j) * 64, 0);
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
  } else if (warp < L::kXfWarp0) {
    // ---- MMA warp of group g: the k-blocks i = g, g + NG, ... of this CTA's
    // sequence, into the group's own accumulator.  Whole warp loops, one
    // elected lane (always the same) issues and commits.
    const int g = warp - L::kMmaWarp0;
    constexpr uint32_t idesc = (1u << 4) | (BF16 ? (1u << 7) | (1u << 10) : 0u) |
                               (static_cast<uint32_t>(BT >> 3) << 17) |
                               (static_cast<uint32_t>(kW4Rows >> 4) << 24);
    const uint32_t a_tmem0 = tmem_base + L::kSlot0 + static_cast<uint32_t>(g * SA * 32);
    const uint64_t b_desc0 = sw128_desc(smem_u32(smem + L::kOffAct));
    int rs = 0, i = 0, jg = 0, seg_i = 0;
    bool ok = true;
    int64_t cur = w4_first(p);
    W4Seg s;
    while (ok && w4_next(p, cur, s)) {
      const int b = seg_i & 1;
      const uint32_t d = tmem_base + static_cast<uint32_t>((b * NG + g) * BT);
      ok = __all_sync(0xffffffffu,
                      mbar_wait(&acc_empty[b], ((seg_i >> 1) & 1) ^ 1u, abort_flag, kSiteMmaTmem, p.status));
      if (!ok) break;
      tc_fence_after();
      uint32_t acc = 0;
      for (int kb = s.kb0; kb < s.kb1 && ok; kb += RK) {
        const int n = s.kb1 - kb < RK ? s.kb1 - kb : RK;
        for (int j = 0; j < n; ++j, ++i) {
          if (i % NG != g) continue;
          const int sl = jg % SA;
          ok = __all_sync(0xffffffffu,
                          mbar_wait(&slot_full[g * SA + sl], (jg / SA) & 1, abort_flag, kSiteMma, p.status));
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            const uint32_t at = a_tmem0 + static_cast<uint32_t>(sl * 32);
            const uint64_t bd = b_desc0 + static_cast<uint32_t>(((rs * RK + j) * L::kAct) >> 4);
            umma_ts_f16(d, at, bd, idesc, acc);
            umma_ts_f16(d, at + 8, bd + 2, idesc, 1u);
            umma_ts_f16(d, at + 16, bd + 4, idesc, 1u);
            umma_ts_f16(d, at + 24, bd + 6, idesc, 1u);
            umma_commit(&slot_empty[g * SA + sl]);
          }
          __syncwarp();
          acc = 1;
          ++jg;
        }
        if (!ok) break;
        // the stage's activation tiles are free once this warp's MMAs are done
        if (elect_one()) umma_commit(&raw_empty[rs]);
        __syncwarp();
        if (++rs == RS) rs = 0;
      }
      if (!ok) break;
      if (elect_one()) umma_commit(&acc_full[b]);
      __syncwarp();
      ++seg_i;
    }
    // Before TMEM is released: every MMA of every group complete.
    if (elect_one()) umma_commit(drain);
    __syncwarp();
    if (g == 0 && lane == 0) {
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < kWaitLimitNs) {
      }
    }
    __syncwarp();
  } else if (warp < kEpiWarp0) {
    // ---- transform, group g of 4 warps; thread = weight row r = TMEM lane r.
    // Each warp dequantizes its 32 rows of a k-block into 32 registers per
    // thread (two 16-bit weights per register, K order) and stores them into
    // the group's TMEM slot with one tcgen05.st; it arrives on the slot's full
    // barrier once its stores have completed.
    const int t = threadIdx.x - 32 * L::kXfWarp0;
    const int g = t >> 7, r = t & 127;
    const uint32_t slot_row = tmem_base + (static_cast<uint32_t>(r & ~31) << 16) + L::kSlot0 +
                              static_cast<uint32_t>(g * SA * 32);
    int rs = 0, i = 0, jg = 0;
    uint32_t rph = 0;
    bool ok = true;
    int64_t cur = w4_first(p);
    W4Seg s;
    while (ok && w4_next(p, cur, s)) {
      for (int kb = s.kb0; kb < s.kb1; kb += RK) {
        const int n = s.kb1 - kb < RK ? s.kb1 - kb : RK;
        const int g_lo = (kb * 64) >> p.gshift;
        ok = __all_sync(0xffffffffu, mbar_wait(&full_raw[rs], rph, abort_flag, kSiteTransform, p.status));
        if (!ok) break;
        const uint32_t words = smem_u32(smem + L::kOffWords + rs * L::kWords) + r * 32;
        const uint32_t grp = smem_u32(smem + L::kOffGrp + rs * L::kGrp) + r * 4;
        for (int j = 0; j < n; ++j, ++i) {
          if (i % NG != g) continue;
          const int sl = jg % SA;
          // loads and dequantization first; the slot wait only gates the TMEM store
          const uint4 wa = lds_v4(words + j * kW4Chunk);
          const uint4 wb = lds_v4(words + j * kW4Chunk + 16);
          const int ga = (((kb + j) * 64) >> p.gshift) - g_lo;
          const int gb = (((kb + j) * 64 + 32) >> p.gshift) - g_lo;
          uint32_t za, sa, zb, sb;
          group_operands<BF16>(lds_u32(grp + ga * kW4Rows * 4), za, sa);
          group_operands<BF16>(lds_u32(grp + gb * kW4Rows * 4), zb, sb);
          uint32_t v[32];
          const uint32_t w8[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const uint4 d4 = dequant_word<BF16>(w8[q], q < 4 ? za : zb, q < 4 ? sa : sb);
            v[4 * q] = d4.x;
            v[4 * q + 1] = d4.y;
            v[4 * q + 2] = d4.z;
            v[4 * q + 3] = d4.w;
          }
          ok = __all_sync(0xffffffffu, mbar_wait(&slot_empty[g * SA + sl], ((jg / SA) & 1) ^ 1u, abort_flag,
                                                 kSiteTransform, p.status));
          if (!ok) break;
          tc_fence_after();  // the slot's previous MMAs have read it
          tmem_st32(slot_row + static_cast<uint32_t>(sl * 32), v);
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&slot_full[g * SA + sl]);
          ++jg;
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[rs]);  // this warp's reads of the stage are over
        if (++rs == RS) {
          rs = 0;
          rph ^= 1u;
        }
      }
    }
  } else {
    // ---- epilogue: TMEM lane = weight row, column = token; sums the NG
    // group accumulators of a segment in group order.  A row tile split
    // across CTAs c_lo..c_hi is finished by c_lo, which covers the tile's
    // first k-blocks at the end of its range; the other CTAs cover it at the
    // start of theirs, publish fp32 slots and bump the tile's arrival
    // counter.  c_lo keeps its own sums in registers, waits (bounded) for the
    // count, adds the slots in CTA order, writes the output and resets the
    // counter to zero for the next call.  Waits only ever point at CTAs of
    // higher index, which finish their part first.
    const int quarter = warp & 3;
    const int rt = quarter * 32 + lane;
    const int e0 = 32 * kEpiWarp0;
    const int me = static_cast<int>(blockIdx.x);
    int seg_i = 0, i0 = 0;
    bool ok = true;
    int64_t cur = w4_first(p);
    W4Seg s;
    while (ok && w4_next(p, cur, s)) {
      const int b = seg_i & 1;
      const int len = s.kb1 - s.kb0;
      ok = bar_and(1, 128, mbar_wait(&acc_full[b], (seg_i >> 1) & 1, abort_flag, kSiteEpilogue, p.status));
      if (!ok) break;
      tc_fence_after();
      const int n = s.tn * kW4Rows + rt;
      const int mc = p.M < BT ? p.M : BT;
      const int64_t u0 = static_cast<int64_t>(s.tn) * p.KB;
      const int c_lo = w4_owner(p.U, p.P, u0), c_hi = w4_owner(p.U, p.P, u0 + p.KB - 1);
      const bool finisher = me == c_lo;
      float y[BT];
#pragma unroll
      for (int j = 0; j < BT; ++j) y[j] = 0.0f;
#pragma unroll
      for (int c0 = 0; c0 < BT; c0 += 16) {
        if (c0 < mc) {
#pragma unroll
          for (int gg = 0; gg < NG; ++gg) {
            // group gg holds k-blocks of this segment iff one is = gg mod NG
            if (len >= NG || (((gg - i0) % NG + NG) % NG) < len) {
              uint32_t v[16];
              tmem_ld16(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                            static_cast<uint32_t>((b * NG + gg) * BT + c0),
                        v);
              tmem_ld_wait16(v);
#pragma unroll
              for (int j = 0; j < 16; ++j) y[c0 + j] = __fadd_rn(y[c0 + j], __uint_as_float(v[j]));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);  // TMEM buffer free for the groups
      if (!finisher) {
        // Publish this CTA's share of the tile (token columns past M are 0).
        float* prow = p.partial + (static_cast<int64_t>(s.slot) * kW4Rows + rt) * BT;
#pragma unroll
        for (int q = 0; q < BT / 4; ++q)
          *reinterpret_cast<float4*>(prow + 4 * q) = make_float4(y[4 * q], y[4 * q + 1], y[4 * q + 2], y[4 * q + 3]);
        __threadfence();
        named_bar_sync(1, 128);
        if (static_cast<int>(threadIdx.x) == e0) atomicAdd(&p.counters[c_lo], 1);
      } else {
        if (c_hi > c_lo) {
          bool arrived = true;
          if (static_cast<int>(threadIdx.x) == e0)
            arrived = wait_count(&p.counters[me], c_hi - c_lo, abort_flag, p.status);
          ok = bar_and(1, 128, arrived);
          if (!ok) break;
          __threadfence();
          for (int c = c_lo + 1; c <= c_hi; ++c) {
            const float4* src =
                reinterpret_cast<const float4*>(p.partial + (static_cast<int64_t>(s.tn + c) * kW4Rows + rt) * BT);
#pragma unroll
            for (int q = 0; q < BT / 4; ++q) {
              const float4 v = __ldcg(src + q);
              y[4 * q] = __fadd_rn(y[4 * q], v.x);
              y[4 * q + 1] = __fadd_rn(y[4 * q + 1], v.y);
              y[4 * q + 2] = __fadd_rn(y[4 * q + 2], v.z);
              y[4 * q + 3] = __fadd_rn(y[4 * q + 3], v.w);
            }
          }
          if (static_cast<int>(threadIdx.x) == e0) p.counters[me] = 0;
        }
        if (n < p.N) {
          const float bias = p.bias != nullptr ? load_as_float(p.bias, p.bias_dtype, n) : 0.0f;
#pragma unroll
          for (int j = 0; j < BT; ++j) {
            if (j < mc) {
              const float o32 = __fadd_rn(y[j], bias);
              uint16_t* o = static_cast<uint16_t*>(p.out) + static_cast<int64_t>(j) * p.ldo + n;
              *o = BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(o32)) : __half_as_ushort(__float2half_rn(o32));
            }
          }
        }
      }
      i0 += len;
      ++seg_i;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == L::kMmaWarp0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// PackedInt4 words (signed nibbles q = u - 8; layout "nk" [N, K/8] or "kn"
// [K/8, N]; element j at nibble j, or 7 - j for order "high") -> W4A16 tiles.
// One thread per output word; rows past N become 0.
__global__ void w4a16_tiles_kernel(const uint32_t* __restrict__ data, int layout_kn, int order_high, int N, int K,
                                   int KB, int64_t total, uint32_t* __restrict__ tiles) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int w = static_cast<int>(i & 7), r = static_cast<int>((i >> 3) & 127);
  const int64_t rest = i >> 10;
  const int kb = static_cast<int>(rest % KB), t = static_cast<int>(rest / KB);
  const int n = t * kW4Rows + r;
  const int64_t kw = static_cast<int64_t>(kb) * 8 + w;
  uint32_t out = 0;
  if (n < N) {
    const uint32_t u = (layout_kn ? data[kw * N + n] : data[static_cast<int64_t>(n) * (K / 8) + kw]) ^ 0x88888888u;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t nib = (u >> (order_high ? 28 - 4 * j : 4 * j)) & 15u;
      out |= nib << (4 * ((j >> 1) + 4 * (j & 1)));
    }
  }
  tiles[i] = out;
}

// PackedInt4 fp32 scales and int32 zeros (zu - 8), [N, G] -> W4A16 group
// operands {s rounded to the 16-bit type (RNE), zu}.  One thread per word.
template <bool BF16>
__global__ void w4a16_groups_kernel(const float* __restrict__ scales, const int32_t* __restrict__ zeros, int N,
                                    int G, int64_t total, uint32_t* __restrict__ groups) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int r = static_cast<int>(i & 127);
  const int64_t rest = i >> 7;
  const int g = static_cast<int>(rest % G), t = static_cast<int>(rest / G);
  const int n = t * kW4Rows + r;
  uint32_t v = 0;
  if (n < N) {
    const int64_t src = static_cast<int64_t>(n) * G + g;
    const float s = scales[src];
    const float z = static_cast<float>(zeros[src] + 8);
    uint32_t sb, zb;
    if constexpr (BF16) {
      sb = __bfloat16_as_ushort(__float2bfloat16_rn(s));
      zb = __bfloat16_as_ushort(__float2bfloat16_rn(z));
    } else {
      sb = __half_as_ushort(__float2half_rn(s));
      zb = __half_as_ushort(__float2half_rn(z));
    }
    v = sb | (zb << 16);
  }
  groups[i] = v;
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

// Activation map: [M rows, K] 16-bit, box 64 x BT, 128-byte swizzle; rows
// past M read as zero.
static cudaError_t act_map(CUtensorMap* map, const void* a, int64_t K, int64_t M, int64_t lda, uint32_t bt) {
  EncodeTiledFn fn = tensor_map_encoder();
  if (fn == nullptr) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(lda * 2)};
  const cuuint32_t box[2] = {64, bt};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(a), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <bool BF16, int BT, int RK, int RS, int XS, int UK>
static cudaError_t launch_w4(const void* a, int64_t lda, const W4Params& p, cudaStream_t stream) {
  using L = W4Layout<BT, RK, RS, XS, UK>;
  auto kernel = w4a16_kernel<BF16, BT, RK, RS, XS, UK>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  CUtensorMap ma;
  cudaError_t e = act_map(&ma, a, p.K, p.M, lda, BT);
  if (e != cudaSuccess) return e;
  kernel<<<p.P, w4_threads<BT, RK, RS, XS, UK>(), L::kAlloc, stream>>>(ma, p);
  return cudaGetLastError();
}

template <bool BF16, int BT, int RK, int RS, int NG>
static cudaError_t launch_w4_decode(const void* a, int64_t lda, const W4Params& p, cudaStream_t stream) {
  using L = W4DecLayout<BT, RK, RS, NG>;
  auto kernel = w4a16_decode_kernel<BF16, BT, RK, RS, NG>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  CUtensorMap ma;
  cudaError_t e = act_map(&ma, a, p.K, p.M, lda, BT);
  if (e != cudaSuccess) return e;
  kernel<<<p.P, L::kThreads, L::kAlloc, stream>>>(ma, p);
  return cudaGetLastError();
}

template <bool BF16, int BT, int RK, int RS, int NG, int SA>
static cudaError_t launch_w4_decode_tm(const void* a, int64_t lda, const W4Params& p, cudaStream_t stream) {
  using L = W4TmLayout<BT, RK, RS, NG, SA>;
  auto kernel = w4a16_decode_tm_kernel<BF16, BT, RK, RS, NG, SA>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  CUtensorMap ma;
  cudaError_t e = act_map(&ma, a, p.K, p.M, lda, BT);
  if (e != cudaSuccess) return e;
  kernel<<<p.P, L::kThreads, L::kAlloc, stream>>>(ma, p);
  return cudaGetLastError();
}

// Decode-kernel selection (M <= 32): 0 = automatic (TMEM operands), 1 = the
// shared-memory-operand kernel, 2 = the TMEM-operand kernel.
static int g_w4_decode_path = 0;
void set_w4a16_path(int path) { g_w4_decode_path = path; }

// Token tile for M tokens; M <= 32 runs stream-K over one token tile.
static int w4_bt(int64_t M) { return M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256; }

struct W4Plan {
  int bt, streamk, P;
  int64_t U;
  size_t workspace;
};

static W4Plan w4_plan(int64_t M, int64_t N, int64_t K) {
  W4Plan pl{};
  pl.bt = w4_bt(M);
  const int64_t T = (N + kW4Rows - 1) / kW4Rows, KB = K / 64;
  const int64_t sms = device_sm_count();
  pl.streamk = pl.bt <= 32;  // decode kernel; larger M runs whole tiles
  if (pl.streamk) {
    pl.U = T * KB;
    pl.P = static_cast<int>(pl.U < sms ? pl.U : sms);
    if (pl.P > kW4MaxCtas) pl.P = kW4MaxCtas;
    pl.workspace = kW4CounterBytes + static_cast<size_t>(T + pl.P - 1) * kW4Rows * pl.bt * 4;
  } else {
    const int64_t tiles = T * ((M + pl.bt - 1) / pl.bt);
    pl.P = static_cast<int>(tiles < sms ? tiles : sms);
  }
  return pl;
}

size_t w4a16_workspace(int64_t M, int64_t N, int64_t K) { return w4_plan(M, N, K).workspace; }

cudaError_t run_w4a16(const void* a, int a_dtype, int64_t lda, const void* tiles, const void* groups, int group,
                      int64_t M, int64_t N, int64_t K, const void* bias, int bias_dtype, void* out, int64_t ldo,
                      float* partial, size_t partial_bytes, cudaStream_t stream) {
  if (M == 0 || N == 0) return cudaSuccess;
  const W4Plan pl = w4_plan(M, N, K);
  if (pl.streamk && (partial == nullptr || partial_bytes < pl.workspace)) return cudaErrorInvalidValue;
  W4Params p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.gshift = group == 32 ? 5 : group == 64 ? 6 : 7;
  p.T = static_cast<int>((N + kW4Rows - 1) / kW4Rows);
  p.KB = static_cast<int>(K / 64);
  p.G = static_cast<int>(K / group);
  p.TM = static_cast<int>((M + pl.bt - 1) / pl.bt);
  p.P = pl.P;
  p.streamk = pl.streamk;
  p.U = pl.U;
  p.tiles = static_cast<const uint8_t*>(tiles);
  p.groups = static_cast<const uint8_t*>(groups);
  p.bias = bias;
  p.bias_dtype = bias_dtype;
  p.out = out;
  p.ldo = ldo;
  p.partial = nullptr;
  p.counters = nullptr;
  if (pl.streamk) {  // counters are zero on entry: zero-filled once, every call leaves them zero
    p.counters = reinterpret_cast<int*>(partial);
    p.partial = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(partial) + kW4CounterBytes);
  }
  p.status = status_word_ptr();
  const bool bf = a_dtype == kBF16;
  cudaError_t e;
  if (pl.streamk) {
    if (g_w4_decode_path == 1) {
      if (pl.bt == 16)
        return bf ? launch_w4_decode<true, 16, 4, 4, 3>(a, lda, p, stream) : launch_w4_decode<false, 16, 4, 4, 3>(a, lda, p, stream);
      return bf ? launch_w4_decode<true, 32, 4, 3, 3>(a, lda, p, stream) : launch_w4_decode<false, 32, 4, 3, 3>(a, lda, p, stream);
    }
    // dequantized k-blocks in TMEM: 4 slots per group at 16 tokens, 3 at 32,
    // and the shared memory they no longer need deepens the raw ring
    if (pl.bt == 16)
      return bf ? launch_w4_decode_tm<true, 16, 4, 7, 3, 4>(a, lda, p, stream)
                : launch_w4_decode_tm<false, 16, 4, 7, 3, 4>(a, lda, p, stream);
    return bf ? launch_w4_decode_tm<true, 32, 4, 6, 3, 3>(a, lda, p, stream)
              : launch_w4_decode_tm<false, 32, 4, 6, 3, 3>(a, lda, p, stream);
  }
  switch (pl.bt) {
#define W4_CASE(BT, RK, RS, XS, UK)                                                                     \
  case BT:                                                                                            \
    e = bf ? launch_w4<true, BT, RK, RS, XS, UK>(a, lda, p, stream) : launch_w4<false, BT, RK, RS, XS, UK>(a, lda, p, stream); \
    break;
    W4_CASE(64, 4, 3, 2, 2)
    W4_CASE(128, 2, 3, 2, 2)
    W4_CASE(256, 1, 5, 2, 1)
#undef W4_CASE
    default: return cudaErrorInvalidValue;
  }
  return e;
}

size_t w4a16_tiles_bytes(int64_t N, int64_t K) {
  return static_cast<size_t>((N + kW4Rows - 1) / kW4Rows) * (K / 64) * kW4Chunk;
}

size_t w4a16_groups_bytes(int64_t N, int64_t K, int group) {
  return static_cast<size_t>((N + kW4Rows - 1) / kW4Rows) * (K / group) * kW4GroupBytes;
}

cudaError_t run_w4a16_prepare(const uint32_t* data, int layout_kn, int order_high, const float* scales,
                              const int32_t* zeros, int64_t N, int64_t K, int group, int dtype, uint32_t* tiles,
                              uint32_t* groups, cudaStream_t stream) {
  const int64_t tw = static_cast<int64_t>(w4a16_tiles_bytes(N, K) / 4);
  const int64_t gw = static_cast<int64_t>(w4a16_groups_bytes(N, K, group) / 4);
  if (tw == 0) return cudaSuccess;
  w4a16_tiles_kernel<<<static_cast<unsigned>((tw + 255) / 256), 256, 0, stream>>>(
      data, layout_kn, order_high, static_cast<int>(N), static_cast<int>(K), static_cast<int>(K / 64), tw, tiles);
  const unsigned gb = static_cast<unsigned>((gw + 255) / 256);
  const int G = static_cast<int>(K / group);
  if (dtype == kBF16) w4a16_groups_kernel<true><<<gb, 256, 0, stream>>>(scales, zeros, static_cast<int>(N), G, gw, groups);
  else w4a16_groups_kernel<false><<<gb, 256, 0, stream>>>(scales, zeros, static_cast<int>(N), G, gw, groups);
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


}  // namespace b2
