// Column-parallel fused linear with the output all-gather folded into the
// GEMM (one process per GPU, weights N-sharded across the ranks of a node).
//
// Each rank computes its N-shard of Y = epilogue(quantize(rotate(x)) @ W.T)
// with the pair TMA-store GEMM, whose epilogue writes every finished output
// unit both to its own full output buffer (TMA store) and, with plain 16-byte
// stores over NVLink, into the same columns of every peer's full output
// buffer.  The transfer therefore overlaps the MMAs tile by tile, and every
// rank ends with the whole row-major Y[M, N_total] -- no separate collective
// and no permute pass.  Completion is signalled per rank through a small
// "gather state" buffer on every GPU: rank r's GEMM releases an epoch number
// into slot r of every rank's flag array once all of its CTAs are done, and
// b2_gather_wait (one tiny kernel) acquires all slots of the local array
// before the stream moves on.  All waits are bounded.
//
// Peer buffers are reached through CUDA IPC (b2_ipc_export / b2_ipc_import);
// no TMA, bulk copy or multicast ever touches peer memory.
#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include "../../include/b2_qlinear.h"
#include "b2_common.cuh"
#include "b2_internal.h"

namespace {

constexpr int kStateBytes = 256;        // flags [0, 32) bytes, counter at 128
constexpr int kCounterOffset = 128;

inline int fail() { return static_cast<int>(cudaErrorInvalidValue); }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn address_range() {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(ptr);
  });
  return fn;
}

// Opened IPC mappings of this process, by handle bytes: one open per
// allocation (a second cudaIpcOpenMemHandle of the same handle fails).
struct Mapping {
  void* base = nullptr;
  int refs = 0;
};
std::mutex g_ipc_mutex;
std::map<std::string, Mapping> g_mappings;

__global__ void gather_wait_kernel(const uint32_t* flags, int world, uint32_t epoch, int* status) {
  const int r = static_cast<int>(threadIdx.x);
  if (r >= world) return;
  const uint64_t start = b2::globaltimer();
  for (uint32_t i = 0;; ++i) {
    const uint32_t v = b2::ld_acquire_sys(flags + r);
    if (static_cast<int32_t>(v - epoch) >= 0) return;  // this epoch or a later one
    if ((i & 255u) == 255u && b2::globaltimer() - start > b2::kWaitLimitNs) {
      if (status != nullptr) atomicCAS(status, 0, 0x100 | b2::kSiteGather);
      return;
    }
    __nanosleep(100);
  }
}

}  // namespace

extern "C" {

size_t b2_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int b2_ipc_export(const void* ptr, void* handle, uint64_t* offset) {
  if (!ptr || !handle || !offset) return fail();
  AddressRangeFn fn = address_range();
  if (fn == nullptr) return static_cast<int>(cudaErrorNotSupported);
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return fail();
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return static_cast<int>(e);
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<uint64_t>(reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base));
  return 0;
}

int b2_ipc_import(const void* handle, uint64_t offset, void** ptr) {
  if (!handle || !ptr) return fail();
  const std::string key(static_cast<const char*>(handle), sizeof(cudaIpcMemHandle_t));
  std::lock_guard<std::mutex> lock(g_ipc_mutex);
  Mapping& m = g_mappings[key];
  if (m.refs == 0) {
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      g_mappings.erase(key);
      return static_cast<int>(e);
    }
    m.base = base;
  }
  ++m.refs;
  *ptr = static_cast<char*>(m.base) + offset;
  return 0;
}

int b2_ipc_release(const void* handle) {
  if (!handle) return fail();
  const std::string key(static_cast<const char*>(handle), sizeof(cudaIpcMemHandle_t));
  std::lock_guard<std::mutex> lock(g_ipc_mutex);
  auto it = g_mappings.find(key);
  if (it == g_mappings.end()) return fail();
  if (--it->second.refs == 0) {
    cudaError_t e = cudaIpcCloseMemHandle(it->second.base);
    g_mappings.erase(it);
    return static_cast<int>(e);
  }
  return 0;
}

size_t b2_gather_state_bytes(void) { return kStateBytes; }

int b2_peer_copy_2d(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width_bytes, int64_t rows,
                    void* stream) {
  if (!dst || !src || width_bytes < 0 || rows < 0 || dpitch < width_bytes || spitch < width_bytes) return fail();
  if (width_bytes == 0 || rows == 0) return 0;
  return static_cast<int>(cudaMemcpy2DAsync(dst, static_cast<size_t>(dpitch), src, static_cast<size_t>(spitch),
                                            static_cast<size_t>(width_bytes), static_cast<size_t>(rows),
                                            cudaMemcpyDefault, static_cast<cudaStream_t>(stream)));
}

int b2_gather_wait(const void* state, int world, uint32_t epoch, void* stream) {
  if (!state || world < 1 || world > b2::kMaxGatherPeers + 1 || epoch == 0) return fail();
  if (reinterpret_cast<uintptr_t>(state) % 256 != 0) return fail();
  gather_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint32_t*>(state), world, epoch, b2::status_word_ptr());
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"

namespace {

// Gather arguments shared by the two gathered GEMM entry points: 0 when the
// output buffers, states and column range are valid.
int check_gather(int world, int rank, int64_t N, int64_t ldc, int64_t col0, int out_dtype, void* const* outs,
                 void* const* states, uint32_t epoch) {
  if (world < 1 || world > b2::kMaxGatherPeers + 1 || rank < 0 || rank >= world) return fail();
  if (!outs || !states || epoch == 0) return fail();
  if (out_dtype != b2::kF16 && out_dtype != b2::kBF16 && out_dtype != b2::kF32) return fail();
  const int ob = out_dtype == b2::kF32 ? 4 : 2;
  if (N % 64 != 0 || col0 < 0 || col0 + N > ldc || (col0 * ob) % 16 != 0 || (ldc * ob) % 16 != 0) return fail();
  for (int q = 0; q < world; ++q) {
    if (!outs[q] || !aligned16(outs[q]) || !states[q]) return fail();
    if (reinterpret_cast<uintptr_t>(states[q]) % 256 != 0) return fail();
  }
  return 0;
}

// Peer outputs (this rank's columns of every other rank's buffer), flag
// slots (peers first, own last), the CTA counter and the epoch.
void fill_gather(b2::GemmParams& p, int world, int rank, int64_t col0, int ob, void* const* outs,
                 void* const* states, uint32_t epoch) {
  p.vec_ok = 1;
  p.gather = 1;
  p.n_peers = 0;
  for (int r = 0; r < world; ++r) {
    if (r == rank) continue;
    p.peer_out[p.n_peers++] = static_cast<char*>(outs[r]) + col0 * ob;
  }
  int slot = 0;
  for (int r = 0; r < world; ++r) {
    if (r == rank) continue;
    p.flag_slot[slot++] = static_cast<uint32_t*>(states[r]) + rank;
  }
  p.flag_slot[slot] = static_cast<uint32_t*>(states[rank]) + rank;
  p.done_count = reinterpret_cast<uint32_t*>(static_cast<char*>(states[rank]) + kCounterOffset);
  p.epoch = epoch;
}

}  // namespace

extern "C" {

int b2_qgemm_gather(int kind, const void* a, int64_t lda, const float* a_scale, const void* w, int64_t ldw,
                    int64_t M, int64_t N, int64_t K, const float* w_scale, int64_t w_scale_count, const void* bias,
                    int bias_dtype, int epilogue, int out_dtype, int64_t ldc, int64_t col0, int world, int rank,
                    void* const* outs, void* const* states, uint32_t epoch, void* stream) {
  if (kind != b2::kKindI8 && kind != b2::kKindE4M3) return fail();
  int st = check_gather(world, rank, N, ldc, col0, out_dtype, outs, states, epoch);
  if (st != 0) return st;
  const int ob = out_dtype == b2::kF32 ? 4 : 2;
  char* own = static_cast<char*>(outs[rank]) + col0 * ob;
  st = b2::check_gemm_args(kind, a, lda, w, ldw, M, N, K, a_scale, w_scale, w_scale_count, bias, bias_dtype,
                           epilogue, own, out_dtype, ldc);
  if (st != 0 || M == 0) return st;
  if (epilogue == b2::kEpiNone) return fail();
  b2::GemmParams p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.sa = a_scale;
  p.sb = w_scale;
  p.sb_scalar = w_scale_count == 1 ? 1 : 0;
  p.bias = bias;
  p.bias_dtype = bias_dtype;
  p.out = own;
  p.out_dtype = out_dtype;
  p.ldc = ldc;
  p.epilogue = epilogue;
  fill_gather(p, world, rank, col0, ob, outs, states, epoch);
  return static_cast<int>(b2::run_qgemm(kind, a, lda, w, ldw, p, 0, static_cast<cudaStream_t>(stream)));
}

int b2_quant_linear_gather(int kind, const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int block,
                           const void* w, int64_t ldw, int64_t N, const float* w_scale, int64_t w_scale_count,
                           const void* bias, int bias_dtype, int epilogue, int out_dtype, int64_t ldc,
                           int64_t col0, int world, int rank, void* const* outs, void* const* states,
                           uint32_t epoch, void* workspace, size_t workspace_bytes, void* stream) {
  int st0 = check_gather(world, rank, N, ldc, col0, out_dtype, outs, states, epoch);
  if (st0 != 0) return st0;
  const int ob = out_dtype == b2::kF32 ? 4 : 2;
  char* own = static_cast<char*>(outs[rank]) + col0 * ob;
  // The fused linear's own argument check, with this rank's columns of its
  // own output as `out`.  M == 0 launches nothing and releases no flag, so
  // callers skip b2_gather_wait for it too.
  int st = b2::check_quant_linear(kind, x, x_dtype, M, K, ldx, block, w, ldw, N, w_scale, w_scale_count, bias,
                                  bias_dtype, epilogue, own, out_dtype, ldc, workspace, workspace_bytes);
  if (st != 0 || M == 0) return st;
  const int64_t ldq = round_up(K, 16);
  uint8_t* q = static_cast<uint8_t*>(workspace);
  float* sa = reinterpret_cast<float*>(q + round_up(M * ldq, 256));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = b2::run_act_quant(x, x_dtype, M, K, ldx, block, kind == b2::kKindE4M3 ? 1 : 0, q, ldq, sa, s,
                                    /*early_dependents=*/true);
  if (e != cudaSuccess) return static_cast<int>(e);
  b2::GemmParams p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.sa = sa;
  p.sb = w_scale;
  p.sb_scalar = w_scale_count == 1 ? 1 : 0;
  p.bias = bias;
  p.bias_dtype = bias_dtype;
  p.out = own;
  p.out_dtype = out_dtype;
  p.ldc = ldc;
  p.epilogue = epilogue;
  p.weight_prefetch = 1;
  fill_gather(p, world, rank, col0, ob, outs, states, epoch);
  return static_cast<int>(b2::run_qgemm(kind, q, ldq, w, ldw, p, 0, s));
}

}  // extern "C"

// ----------------------------------------------- copy-engine gather variant
// The same column-parallel linear with the transfer done by the copy engines:
// the linear runs in M-chunks on the caller's stream (prologue + plain pair
// GEMM into this rank's columns of its own output); after each chunk, one
// 2-D copy per peer, on a per-peer copy stream, carries the chunk's block
// into that peer's output while the next chunk is multiplied.  When a peer's
// copies are done a one-thread kernel on the same copy stream increments
// this rank's count slot in the peer's state (system-scope release).  The
// caller's stream then joins the copy streams and runs a bounded wait until
// every peer's count reaches this call's sequence number, which the wait
// kernel itself advances -- so nothing on the host depends on a per-call
// value and a whole step can be captured in a CUDA graph and replayed.
// The wait is its own entry point (b2_gather_wait_ce), enqueued after the
// call; calls on one device must not overlap (they share the copy streams).
namespace {

constexpr int kCeCountOffset = 32;     // uint32 counts [world] (bytes 32..63)
constexpr int kCeSeqOffset = 160;      // this rank's call sequence number
constexpr int kCeMaxChunks = 8;

struct CeStreams {
  bool ready = false;
  cudaStream_t copy[b2::kMaxGatherPeers];
  cudaEvent_t chunk[kCeMaxChunks];
  cudaEvent_t done[b2::kMaxGatherPeers];
};
CeStreams g_ce[64];
std::mutex g_ce_mutex;

cudaError_t ce_streams(CeStreams** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_ce_mutex);
  CeStreams& c = g_ce[dev];
  if (!c.ready) {
    for (int i = 0; i < b2::kMaxGatherPeers; ++i) {
      if ((e = cudaStreamCreateWithFlags(&c.copy[i], cudaStreamNonBlocking)) != cudaSuccess) return e;
      if ((e = cudaEventCreateWithFlags(&c.done[i], cudaEventDisableTiming)) != cudaSuccess) return e;
    }
    for (int i = 0; i < kCeMaxChunks; ++i)
      if ((e = cudaEventCreateWithFlags(&c.chunk[i], cudaEventDisableTiming)) != cudaSuccess) return e;
    c.ready = true;
  }
  *out = &c;
  return cudaSuccess;
}

__global__ void ce_signal_kernel(uint32_t* count_slot) {
  __threadfence_system();
  asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(count_slot) : "memory");
}

__global__ void ce_wait_kernel(uint32_t* state, int world, int rank, int* status) {
  uint32_t* seq_slot = reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(state) + kCeSeqOffset);
  const uint32_t* counts = reinterpret_cast<const uint32_t*>(reinterpret_cast<char*>(state) + kCeCountOffset);
  const uint32_t seq = *seq_slot + 1u;  // only this kernel writes the slot, one launch at a time per stream
  __syncthreads();
  if (threadIdx.x == 0) *seq_slot = seq;
  const int r = static_cast<int>(threadIdx.x);
  if (r >= world || r == rank) return;
  const uint64_t start = b2::globaltimer();
  for (uint32_t i = 0;; ++i) {
    if (static_cast<int32_t>(b2::ld_acquire_sys(counts + r) - seq) >= 0) return;
    if ((i & 255u) == 255u && b2::globaltimer() - start > b2::kWaitLimitNs) {
      if (status != nullptr) atomicCAS(status, 0, 0x100 | b2::kSiteGather);
      return;
    }
    __nanosleep(100);
  }
}

}  // namespace

extern "C" int b2_quant_linear_gather_ce(int kind, const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx,
                                         int block, const void* w, int64_t ldw, int64_t N, const float* w_scale,
                                         int64_t w_scale_count, const void* bias, int bias_dtype, int epilogue,
                                         int out_dtype, int64_t ldc, int64_t col0, int world, int rank,
                                         void* const* outs, void* const* states, int chunks, void* workspace,
                                         size_t workspace_bytes, void* stream) {
  if (world < 1 || world > b2::kMaxGatherPeers + 1 || rank < 0 || rank >= world) return fail();
  if (!outs || !states || chunks < 1 || chunks > kCeMaxChunks) return fail();
  if (out_dtype != b2::kF16 && out_dtype != b2::kBF16 && out_dtype != b2::kF32) return fail();
  const int ob = out_dtype == b2::kF32 ? 4 : 2;
  if (col0 < 0 || col0 + N > ldc || (col0 * ob) % 16 != 0 || (ldc * ob) % 16 != 0) return fail();
  for (int q = 0; q < world; ++q) {
    if (!outs[q] || !aligned16(outs[q]) || !states[q]) return fail();
    if (reinterpret_cast<uintptr_t>(states[q]) % 256 != 0) return fail();
  }
  char* own = static_cast<char*>(outs[rank]) + col0 * ob;
  int st = b2::check_quant_linear(kind, x, x_dtype, M, K, ldx, block, w, ldw, N, w_scale, w_scale_count, bias,
                                  bias_dtype, epilogue, own, out_dtype, ldc, workspace, workspace_bytes);
  if (st != 0 || M == 0) return st;
  CeStreams* cs = nullptr;
  cudaError_t e = ce_streams(&cs);
  if (e != cudaSuccess) return static_cast<int>(e);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t ldq = round_up(K, 16);
  uint8_t* q = static_cast<uint8_t*>(workspace);
  float* sa = reinterpret_cast<float*>(q + round_up(M * ldq, 256));
  const int eb = x_dtype == b2::kF32 ? 4 : 2;
  // chunks of whole 256-row pair tiles
  int64_t rows = round_up((M + chunks - 1) / chunks, 256);
  for (int64_t m0 = 0, c = 0; m0 < M; m0 += rows, ++c) {
    const int64_t mc = M - m0 < rows ? M - m0 : rows;
    e = b2::run_act_quant(static_cast<const char*>(x) + m0 * ldx * eb, x_dtype, mc, K, ldx, block,
                          kind == b2::kKindE4M3 ? 1 : 0, q + m0 * ldq, ldq, sa + m0, s, /*early_dependents=*/true);
    if (e != cudaSuccess) return static_cast<int>(e);
    b2::GemmParams p{};
    p.M = static_cast<int>(mc);
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.sa = sa + m0;
    p.sb = w_scale;
    p.sb_scalar = w_scale_count == 1 ? 1 : 0;
    p.bias = bias;
    p.bias_dtype = bias_dtype;
    p.out = own + m0 * ldc * ob;
    p.out_dtype = out_dtype;
    p.ldc = ldc;
    p.epilogue = epilogue;
    p.vec_ok = 1;
    p.weight_prefetch = 1;
    if ((e = b2::run_qgemm(kind, q + m0 * ldq, ldq, w, ldw, p, 0, s)) != cudaSuccess) return static_cast<int>(e);
    if (world == 1) continue;
    if ((e = cudaEventRecord(cs->chunk[c], s)) != cudaSuccess) return static_cast<int>(e);
    for (int r = 0, j = 0; r < world; ++r) {
      if (r == rank) continue;
      cudaStream_t cp = cs->copy[j++];
      if ((e = cudaStreamWaitEvent(cp, cs->chunk[c], 0)) != cudaSuccess) return static_cast<int>(e);
      char* dst = static_cast<char*>(outs[r]) + (m0 * ldc + col0) * ob;
      if ((e = cudaMemcpy2DAsync(dst, static_cast<size_t>(ldc * ob), own + m0 * ldc * ob, static_cast<size_t>(ldc * ob),
                                 static_cast<size_t>(N * ob), static_cast<size_t>(mc), cudaMemcpyDefault, cp)) !=
          cudaSuccess)
        return static_cast<int>(e);
    }
  }
  if (world > 1) {
    for (int r = 0, j = 0; r < world; ++r) {
      if (r == rank) continue;
      cudaStream_t cp = cs->copy[j];
      uint32_t* slot = reinterpret_cast<uint32_t*>(static_cast<char*>(states[r]) + kCeCountOffset) + rank;
      ce_signal_kernel<<<1, 1, 0, cp>>>(slot);
      if ((e = cudaGetLastError()) != cudaSuccess) return static_cast<int>(e);
      if ((e = cudaEventRecord(cs->done[j], cp)) != cudaSuccess) return static_cast<int>(e);
      if ((e = cudaStreamWaitEvent(s, cs->done[j], 0)) != cudaSuccess) return static_cast<int>(e);
      ++j;
    }
  }
  return 0;
}

extern "C" int b2_gather_wait_ce(void* state, int world, int rank, void* stream) {
  if (!state || world < 1 || world > b2::kMaxGatherPeers + 1 || rank < 0 || rank >= world) return fail();
  if (reinterpret_cast<uintptr_t>(state) % 256 != 0) return fail();
  ce_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<uint32_t*>(state), world, rank,
                                                                  b2::status_word_ptr());
  return static_cast<int>(cudaGetLastError());
}

// ------------------------------------ column-parallel INT8 activation exchange
// For a stack of column-parallel layers, the next layer's input is gathered
// as INT8 codes instead of fp16 outputs (half the bytes): each rank rotates
// and reduces its own column slice of the layer output (whole rotation
// blocks), the per-row absmax slices are exchanged (b2_shard_amax), and each
// rank quantizes its slice with the row's global scale straight into every
// rank's code buffer (b2_shard_codes).  Each phase ends by releasing `epoch`
// into slot `rank` of every rank's state; b2_gather_wait on the local state
// (one per phase) is the barrier before the next phase / the next GEMM.
namespace {

int shard_checks(const void* y, int y_dtype, int64_t M, int64_t Ns, int64_t ldy, int block, int world, int rank,
                 void* const* states, uint32_t epoch) {
  if (world < 1 || world > b2::kMaxGatherPeers + 1 || rank < 0 || rank >= world) return fail();
  if (!states || epoch == 0 || M < 0 || M > INT32_MAX || Ns < 0 || Ns % 64 != 0 || Ns / 64 > 384) return fail();
  if (y_dtype != b2::kF16 && y_dtype != b2::kBF16 && y_dtype != b2::kF32) return fail();
  if (block > 1 && ((block & (block - 1)) != 0 || block > 2048 || (Ns > 0 && Ns % block != 0))) return fail();
  if (block < 0) return fail();
  const int eb = y_dtype == b2::kF32 ? 4 : 2;
  if (Ns > 0 && M > 0 && (!y || !aligned16(y) || ldy < Ns || (ldy * eb) % 16 != 0)) return fail();
  for (int q = 0; q < world; ++q)
    if (!states[q] || reinterpret_cast<uintptr_t>(states[q]) % 256 != 0) return fail();
  return 0;
}

void shard_signal_args(b2::ShardArgs& sh, int world, int rank, void* const* states, uint32_t epoch) {
  sh.world = world;
  sh.rank = rank;
  for (int q = 0; q < world; ++q) sh.flag_slot[q] = static_cast<uint32_t*>(states[q]) + rank;
  sh.done_count = reinterpret_cast<uint32_t*>(static_cast<char*>(states[rank]) + kCounterOffset);
  sh.epoch = epoch;
}

}  // namespace

extern "C" int b2_shard_amax(const void* y, int y_dtype, int64_t M, int64_t Ns, int64_t ldy, int block, int world,
                             int rank, void* const* xchg, void* const* states, uint32_t epoch, void* stream) {
  int st = shard_checks(y, y_dtype, M, Ns, ldy, block, world, rank, states, epoch);
  if (st != 0) return st;
  if (!xchg) return fail();
  for (int q = 0; q < world; ++q)
    if (!xchg[q] || reinterpret_cast<uintptr_t>(xchg[q]) % 4 != 0) return fail();
  if (M == 0) return 0;
  b2::ShardArgs sh;
  shard_signal_args(sh, world, rank, states, epoch);
  for (int q = 0; q < world; ++q) sh.xchg[q] = static_cast<float*>(xchg[q]);
  return static_cast<int>(b2::run_shard_quant(1, y, y_dtype, M, Ns, ldy, block, 0, 0, nullptr, sh,
                                              static_cast<cudaStream_t>(stream)));
}

extern "C" int b2_shard_codes(const void* y, int y_dtype, int64_t M, int64_t Ns, int64_t ldy, int block, int quant,
                              int world, int rank, const void* xchg_local, void* const* q_outs, int64_t ldq,
                              int64_t col0, float* scale, void* const* states, uint32_t epoch, void* stream) {
  int st = shard_checks(y, y_dtype, M, Ns, ldy, block, world, rank, states, epoch);
  if (st != 0) return st;
  if (quant != 0 && quant != 1) return fail();
  if (!xchg_local || reinterpret_cast<uintptr_t>(xchg_local) % 4 != 0 || !q_outs || !scale) return fail();
  if (reinterpret_cast<uintptr_t>(scale) % 4 != 0 || col0 < 0 || ldq % 16 != 0 || col0 % 16 != 0 ||
      col0 + Ns > ldq)
    return fail();
  for (int q = 0; q < world; ++q)
    if (!q_outs[q] || !aligned16(q_outs[q])) return fail();
  if (M == 0) return 0;
  b2::ShardArgs sh;
  shard_signal_args(sh, world, rank, states, epoch);
  sh.xlocal = static_cast<const float*>(xchg_local);
  for (int q = 0; q < world; ++q) sh.qout[q] = static_cast<uint8_t*>(q_outs[q]) + col0;
  return static_cast<int>(b2::run_shard_quant(2, y, y_dtype, M, Ns, ldy, block, quant, ldq, scale, sh,
                                              static_cast<cudaStream_t>(stream)));
}

// Both exchange phases in one cooperative launch: the absmax pass, an
// in-kernel barrier on every rank's absmax flags (bounded), then the codes
// pass.  A rank whose slice is empty runs the two-launch form instead.
extern "C" int b2_shard_exchange(const void* y, int y_dtype, int64_t M, int64_t Ns, int64_t ldy, int block,
                                 int quant, int world, int rank, void* const* xchg, void* const* amax_states,
                                 uint32_t epoch_amax, void* const* q_outs, int64_t ldq, int64_t col0, float* scale,
                                 void* const* code_states, uint32_t epoch_codes, void* stream) {
  int st = shard_checks(y, y_dtype, M, Ns, ldy, block, world, rank, amax_states, epoch_amax);
  if (st == 0) st = shard_checks(y, y_dtype, M, Ns, ldy, block, world, rank, code_states, epoch_codes);
  if (st != 0) return st;
  if (quant != 0 && quant != 1) return fail();
  if (!xchg || !q_outs || !scale || reinterpret_cast<uintptr_t>(scale) % 4 != 0) return fail();
  if (col0 < 0 || ldq % 16 != 0 || col0 % 16 != 0 || col0 + Ns > ldq) return fail();
  for (int q = 0; q < world; ++q) {
    if (!xchg[q] || reinterpret_cast<uintptr_t>(xchg[q]) % 4 != 0) return fail();
    if (!q_outs[q] || !aligned16(q_outs[q])) return fail();
  }
  if (M == 0) return 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (Ns == 0) {
    st = b2_shard_amax(y, y_dtype, M, Ns, ldy, block, world, rank, xchg, amax_states, epoch_amax, stream);
    if (st == 0) st = b2_gather_wait(amax_states[rank], world, epoch_amax, stream);
    if (st == 0)
      st = b2_shard_codes(y, y_dtype, M, Ns, ldy, block, quant, world, rank, xchg[rank], q_outs, ldq, col0, scale,
                          code_states, epoch_codes, stream);
    return st;
  }
  b2::ShardArgs sh;
  shard_signal_args(sh, world, rank, amax_states, epoch_amax);
  for (int q = 0; q < world; ++q) {
    sh.xchg[q] = static_cast<float*>(xchg[q]);
    sh.qout[q] = static_cast<uint8_t*>(q_outs[q]) + col0;
    sh.flag_slot2[q] = static_cast<uint32_t*>(code_states[q]) + rank;
  }
  sh.xlocal = static_cast<const float*>(xchg[rank]);
  sh.own_flags = static_cast<const uint32_t*>(amax_states[rank]);
  sh.done_count2 = reinterpret_cast<uint32_t*>(static_cast<char*>(code_states[rank]) + kCounterOffset);
  sh.epoch2 = epoch_codes;
  sh.status = b2::status_word_ptr();
  return static_cast<int>(b2::run_shard_quant(3, y, y_dtype, M, Ns, ldy, block, quant, ldq, scale, sh, s));
}
