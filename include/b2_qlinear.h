/*
 * b2_qlinear.h -- C ABI of the B200 (sm_100a) quantized-linear library
 * (librdna2_b200.so).  Plain pointers, sizes and dtype codes; no framework
 * types.  Conventions follow the reference's native ABI precedent
 * (rdna2-ops/kernels.hip:283-319, `rdna2_group_norm_silu`):
 *   - every entry point returns an int that is a cudaError_t value (0 = ok);
 *   - work is enqueued asynchronously on the caller's stream (`void* stream`,
 *     a cudaStream_t; NULL = legacy default stream);
 *   - the caller owns and allocates every output and workspace buffer;
 *     entry points never allocate device memory and never synchronize
 *     (except b2_device_status, which is documented as synchronous);
 *   - all device pointers belong to the current CUDA device.
 *
 * dtype codes:  0 = float32, 1 = float16, 2 = bfloat16, 3 = int32,
 *               4 = float8 e4m3fn, 5 = float8 e5m2 (activation-prologue inputs)
 * epilogue:     0 = separate  v = float(acc)*(sa*sb) [+ bias] in fp32, then cast
 *                               (rdna2_ops/int8_gemm.py:53-63, rounding="separate")
 *               1 = fma       v = fma(float(acc), sa*sb, bias)  (rounding="fused")
 *               2 = kitchen   y = cast(float(acc)*(sa*sb)); y = cast(y + cast(bias))
 *                               (production/MOSS_RDNA2_INT8/backend.py:128-143)
 *               3 = none      raw int32 accumulator (out_dtype must be 3)
 * kind:         0 = int8 x int8 -> int32 (tcgen05 kind::i8)
 *               1 = e4m3 x e4m3 -> fp32  (tcgen05 kind::f8f6f4)
 *               2 = bf16 x bf16 -> fp32  (tcgen05 kind::f16)
 *               3 = fp16 x fp16 -> fp32  (tcgen05 kind::f16)
 */
#ifndef B2_QLINEAR_H_
#define B2_QLINEAR_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Library ABI version (increments on any signature change). */
int b2_version(void);

/* Human-readable text for a status code returned by any entry point. */
const char* b2_error_string(int status);

/* Number of SMs the persistent kernels size their grid to on the current
 * device. */
int b2_sm_count(void);

/* Number of 2-CTA clusters of the pair GEMM kernel that fit on the current
 * device at once (its persistent grid, in pairs), or -1 when cluster launch
 * is unavailable. */
int b2_pair_capacity(void);

/* Process-wide GEMM kernel selection: 0 = automatic (pair or single tiles by
 * a persistent-wave time model), 1 = single-CTA kernel, 2 = pair kernel (both
 * with automatic N tile), 3 = single N=256, 4 = single N=128, 5 = pair
 * N=256, 6 = pair N=192, 7 = pair N=256 with the output staged in shared
 * memory and written by TMA stores (automatic choice for pair tiles whose
 * output rows are 16-byte aligned; 5 otherwise), 8 = split-K: M <= 32 only
 * (automatic there), 128-row swap-AB weight tiles split along K over the
 * CTAs of a thread-block cluster and reduced in the leader's shared memory.
 * A tuning and verification knob; INT8 results are identical for every
 * choice, floating kinds differ only in fp32 summation order; 9 = pair N=192
 * with the TMA-store epilogue (6 for unaligned outputs).
 * No reference counterpart (the reference exposes tile keywords instead,
 * rdna2_ops/int8_gemm.py:195-214). */
int b2_set_gemm_path(int path);

/* Process-wide activation-prologue kernel selection: 0 = automatic (the
 * lane-block kernel where it applies), 1 = the warp-shuffle kernel (every
 * mode), 2 = the lane-block kernel: one lane per 64 elements, INT8
 * ties-to-even codes of fp32/fp16/bf16 rows with K % 64 == 0, rotation
 * blocks <= 2048 and 16-byte aligned input and code rows (other
 * calls fall back to 1).  A tuning and verification knob; codes and scales
 * are identical for every choice.  No reference counterpart. */
int b2_set_prologue_path(int path);

/* Process-wide W4A16 decode-kernel selection (M <= 32): 0 = automatic (the
 * kernel that keeps dequantized weights in tensor memory), 1 = the kernel
 * that stages them in shared memory, 2 = tensor memory.  A tuning and
 * verification knob: both dequantize identically and differ only in the
 * tensor core's fp32 summation order.  No reference counterpart. */
int b2_set_w4a16_path(int path);

/* Process-wide transport of the fused column-parallel gather
 * (b2_quant_linear_gather): 0 = default (2), 1 = each staged 32-row output
 * unit copied to every peer by 16-byte SM stores from the epilogue warps,
 * 2 = by TMA stores through one tensor map per peer output.  Outputs,
 * flags and completion rules are identical for every choice.  No reference
 * counterpart. */
int b2_set_gather_store(int mode);

/* SYNCHRONOUS: read (and if reset != 0 clear) the device status word that a
 * kernel sets when one of its bounded waits gives up (0 = no failure; else
 * 0x100 | site).  Call after synchronizing the stream. */
int b2_device_status(int* status, int reset);

/* Activation prologue: optional block-Hadamard rotation, per-row absmax,
 * round-to-nearest-even quantization.
 *   x      [M,K] of x_dtype (0/1/2, or fp8 4/5), row stride ldx elements
 *   block  0 or 1 = no rotation; else a power of two dividing K (<= 4096)
 *   quant  0 = int8 (scale = absmax/127, round half even, codes in [-127,127]);
 *          1 = e4m3 (scale = absmax/448, saturating);
 *          2 = int8 with the reference row quantizer's rounding
 *              (rdna2_ops/fp8_weight_gemm_v06.py:87-90: step = max(absmax/127,
 *              1e-20), floor(z + 0.5) / ceil(z - 0.5) in fp32)
 *   q      [M,K] 1-byte codes, row stride ldq bytes (columns >= K untouched)
 *   scale  [M] fp32
 * Replaces Kitchen's _rotate_activation + quantize_int8_rowwise at
 * production/MOSS_RDNA2_INT8/backend.py:112-122 and rdna2_ops/int8_gemm.py:249-255,
 * and the row quantizer rdna2_ops/fp8_weight_gemm_v06.py:76-92. */
int b2_act_quant(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int block,
                 int quant, void* q, int64_t ldq, float* scale, void* stream);

/* Quantized GEMM with fused epilogue: out[m,n] = epi(sum_k a[m,k]*b[n,k]).
 *   a       [M,K] K-major, row stride lda elements, 16-byte aligned base,
 *           lda*elem a multiple of 16
 *   b       [N,K] K-major (the weight as stored), same alignment rules
 *   a_scale [M] fp32 (NULL only with epilogue 3)
 *   b_scale [N] fp32 or a single fp32 when b_scale_count == 1
 *   bias    [N] of bias_dtype (0/1/2) or NULL
 *   out     [M,N] of out_dtype, row stride ldc elements
 * Replaces rdna2_ops/int8_gemm.py:152-214 (int8_matmul, int8_gemm_dequant,
 * kernel _int8_dot_dequant at :19-67).  Requires K <= 131071 for kind 0. */
int b2_qgemm(int kind, const void* a, int64_t lda, const void* b, int64_t ldb, int64_t M,
             int64_t N, int64_t K, const float* a_scale, const float* b_scale,
             int64_t b_scale_count, const void* bias, int bias_dtype, int epilogue, void* out,
             int out_dtype, int64_t ldc, void* stream);

/* Strided -> K-major copy used for operand views the TMA cannot read
 * directly (odd strides, transposed [K,N] weights):
 *   dst[r*ldd + c] = src[r*s_row + c*s_col] for c < cols, 0 for cols <= c < ldd.
 * elem_bytes 1 or 2; strides in elements.  Serves the stride-aware contract of
 * rdna2_ops/int8_gemm.py:39-40 for layouts outside the fast path. */
int b2_repack(const void* src, int elem_bytes, int64_t rows, int64_t cols, int64_t s_row,
              int64_t s_col, void* dst, int64_t ldd, void* stream);

/* Workspace bytes b2_quant_linear needs for an [M,K] activation. */
size_t b2_quant_linear_workspace_bytes(int64_t M, int64_t K);

/* Fused quantized linear: act_quant (rotation + per-token quantization of x)
 * followed by b2_qgemm against a pre-quantized weight.
 *   kind 0: W8A8 INT8 (w int8 [N,K]); kind 1: FP8 (w e4m3 [N,K])
 *   w_scale [N] fp32 or one fp32 (w_scale_count 1)
 *   workspace >= b2_quant_linear_workspace_bytes(M, K), 256-byte aligned
 * Replaces production/MOSS_RDNA2_INT8/backend.py:71-145 (int8_linear) and
 * rdna2_ops/int8_gemm.py:231-263 (moss_int8_gemm_candidate's candidate). */
int b2_quant_linear(int kind, const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx,
                    int block, const void* w, int64_t ldw, int64_t N, const float* w_scale,
                    int64_t w_scale_count, const void* bias, int bias_dtype, int epilogue,
                    void* out, int out_dtype, int64_t ldc, void* workspace,
                    size_t workspace_bytes, void* stream);

/* W4A16 weight format ("tiles"), a caller-owned pack of one PackedInt4
 * (the reference keeps packs caller-owned, int4_weight_gemm_v07.py:4-6):
 *   tiles   u32 [T][K/64][128][8], T = ceil(N/128): one 4 KiB chunk per
 *           (128-row tile, 64-element k-block), unsigned nibbles u = q + 8;
 *           element j = k % 8 of a word at nibble (j >> 1) + 4*(j & 1)
 *   groups  u32 [T][K/group][128]: low 16 bits the scale, high 16 bits the
 *           zero point zu (integer 0..15), both in the activation's type
 * Rows past N are zero.  The byte sizes of the two buffers: */
size_t b2_w4a16_tiles_bytes(int64_t N, int64_t K);
size_t b2_w4a16_groups_bytes(int64_t N, int64_t K, int group);

/* PackedInt4 (int4_weight_gemm_v07.py:20-46: data int32 signed nibbles
 * q = u - 8, layout_kn 0 "nk" [N,K/8] / 1 "kn" [K/8,N], order_high 1 puts
 * element 0 in the top nibble; scales fp32 [N,K/group]; zeros int32
 * zu - 8 [N,K/group]) -> tiles + groups for activations of dtype (1 fp16,
 * 2 bf16).  Lossless except the scale's round-to-nearest-even cast to
 * 16 bits, the one rounding the 16-bit scale format implies. */
int b2_w4a16_prepare(const void* data, int layout_kn, int order_high, const float* scales,
                     const void* zeros, int64_t N, int64_t K, int group, int dtype, void* tiles,
                     void* groups, void* stream);

/* Workspace bytes b2_w4a16_gemm needs for these sizes on the current device
 * (0 = none; M <= 32 needs one, sized by the SM count).  Its first 4 KiB
 * are arrival counters: zero-fill them once before the first use; every
 * completed call leaves them zero again, for any later shape (after a call
 * that left a nonzero b2_device_status, zero them again). */
size_t b2_w4a16_workspace_bytes(int64_t M, int64_t N, int64_t K, int group);

/* W4A16 weight-only GEMM: out[m,n] = sum_k a[m,k] * w[n,k] (+ bias[n]) with
 * w[n,k] = round((u - zu) * s) in the activation's 16-bit type.
 *   a       [M,K] fp16 (a_dtype 1) or bf16 (2), row stride lda, 16-byte rows
 *   tiles, groups  from b2_w4a16_prepare (16-byte aligned)
 *   group   32, 64 or 128; K a multiple of 64 and of group
 *   out     [M,N] in a_dtype, row stride ldo; bias [N] of bias_dtype or NULL
 *   workspace >= b2_w4a16_workspace_bytes(M, N, K, group), 16-byte aligned,
 *           zero-filled before its first use (see above); calls sharing
 *           one workspace must not overlap on the GPU
 * Results are deterministic run to run on one device.  Replaces
 * int4_linear_a16 / _linear_dot2 (rdna2_ops/int4_weight_gemm_v07.py
 * :540-564, 365-387) with uint4 + 16-bit scales/zero points. */
int b2_w4a16_gemm(const void* a, int a_dtype, int64_t lda, const void* tiles, const void* groups,
                  int group, int64_t M, int64_t N, int64_t K, const void* bias, int bias_dtype,
                  void* out, int64_t ldo, void* workspace, size_t workspace_bytes, void* stream);

/* W4A8 grouped linear (int4_linear_a8, rdna2_ops/int4_weight_gemm_v07.py
 * :476-537; float order of int4_model_switches_v07.py:19-34
 * grouped_integer_reference): for each group g an exact integer dot
 * e_g = sum a[m,k] * (q - z), total = total + fp32(e_g) * s[n,g] in group
 * order (product and sum each rounded), y = total * a_scale[m] (+ bias[n]),
 * fp32 out; integer != 0 writes sum_g e_g as int32 instead (bias and scales
 * unused).  Weight format from b2_w4a8_prepare (a caller-owned pack of one
 * PackedInt4):
 *   tiles   u64 [ceil(N/128)][K/128][8][128] unsigned nibbles u = q + 8
 *   groups  u64 [ceil(N/128)][K/group][128] = {fp32 scale, zu = z + 8}
 * K a multiple of 128; group 32, 64 or 128. */
size_t b2_w4a8_tiles_bytes(int64_t N, int64_t K);
size_t b2_w4a8_groups_bytes(int64_t N, int64_t K, int group);
int b2_w4a8_prepare(const void* data, int layout_kn, int order_high, const float* scales, const void* zeros,
                    int64_t N, int64_t K, int group, void* tiles, void* groups, void* stream);
/* Workspace (per-group activation sums) for b2_w4a8_gemm; rewritten every call. */
size_t b2_w4a8_workspace_bytes(int64_t M, int64_t K, int group);
/*   a        int8 [M,K], row stride lda bytes (multiple of 16), 16-byte aligned
 *   a_scale  fp32 [M]; bias [N] of bias_dtype (0/1/2) or NULL
 *   out      fp32 (integer: int32) [M, ldo] */
int b2_w4a8_gemm(const void* a, int64_t lda, const void* tiles, const void* groups, int group, int64_t M,
                 int64_t N, int64_t K, const float* a_scale, const void* bias, int bias_dtype, int integer,
                 void* out, int64_t ldo, void* workspace, size_t workspace_bytes, void* stream);

/* Exact fp8 decode (rdna2_ops/fp8_weight_gemm_v06.py:22-46, 109-124):
 * w [rows, cols] of fp8_dtype (4 e4m3fn, 5 e5m2), row stride ld bytes ->
 * out of out_dtype (0 fp32, 1 fp16), row stride ldo elements. */
int b2_fp8_decode(const void* w, int fp8_dtype, int64_t rows, int64_t cols, int64_t ld, int out_dtype,
                  void* out, int64_t ldo, void* stream);

/* Group INT4 packer with the semantics of pack_int4 / pack_int4_cpu
 * (rdna2_ops/int4_weight_gemm_v07.py:49-82, 413-430): w [N,K] of w_dtype
 * (0/1/2), row stride ldw; outputs PackedInt4 storage -- data int32 words
 * (layout_kn 0: [N,K/8], 1: [K/8,N]; order_high puts element 0 in the top
 * nibble), scales fp32 [N,K/group], zeros int32 (zu - 8), sums int32. */
int b2_pack_int4(const void* w, int w_dtype, int64_t ldw, int64_t N, int64_t K, int group,
                 int symmetric, int layout_kn, int order_high, void* data, float* scales,
                 void* zeros, void* sums, void* stream);

/* Decode PackedInt4 storage (rdna2_ops/int4_weight_gemm_v07.py:433-441):
 * out_dtype 0 = fp32 (q - z) * s, 1 = fp16 of the same, 3 = int8 q - z. */
int b2_unpack_int4(const void* data, int layout_kn, int order_high, const float* scales,
                   const void* zeros, int64_t N, int64_t K, int group, int out_dtype, void* out,
                   void* stream);

/* ---- Column-parallel linear with the output gather fused into the GEMM ----
 * One process per GPU; the weight is N-sharded across `world` ranks and every
 * rank holds a full output buffer Y[M, ldc] plus a gather-state buffer of
 * b2_gather_state_bytes() bytes (256-byte aligned, zero-filled once before
 * first use).  Each rank maps its peers' output and state buffers into its own
 * address space with the IPC helpers below.  Replaces the multi-GPU
 * reassembly of the per-layer linear production/MOSS_RDNA2_INT8/backend.py
 * :112-145 (the reference itself is single-GPU), i.e. ColumnParallelLinear's
 * NCCL all-gather of the shard outputs.
 *
 * b2_ipc_export: handle (b2_ipc_handle_bytes() bytes) and byte offset of the
 *   device allocation holding `ptr` (cudaIpcGetMemHandle of its base).
 * b2_ipc_import: map a peer's exported allocation into this process (peer
 *   access enabled lazily); *ptr = mapped base + offset.  Reference counted per
 *   handle; b2_ipc_release drops one reference and unmaps at zero. */
size_t b2_ipc_handle_bytes(void);
int b2_ipc_export(const void* ptr, void* handle, uint64_t* offset);
int b2_ipc_import(const void* handle, uint64_t offset, void** ptr);
int b2_ipc_release(const void* handle);
size_t b2_gather_state_bytes(void);

/* The fused linear of b2_quant_linear for this rank's shard (w [N,K], w_scale,
 * bias: the shard's rows), with the epilogue writing each output tile into
 * columns [col0, col0 + N) of EVERY rank's output: outs[r] = rank r's full
 * output buffer as mapped here (outs[rank] the local one), states[r] = rank
 * r's gather-state buffer as mapped here.  Peer copies are plain 16-byte
 * stores over NVLink issued while later tiles are still being multiplied.
 * When all of this rank's work is stored, `epoch` (nonzero, increasing per
 * call) is released into slot `rank` of every rank's state.  Requires
 * N % 64 == 0, 16-byte aligned output rows and columns (col0, ldc), kind 0/1.
 * M == 0 launches nothing and releases nothing.  Output buffers are written by
 * every rank: a consumer may read Y only after b2_gather_wait for the epoch,
 * and a rank may start the next call writing the same buffer only after every
 * rank has finished reading it (alternate two buffers between layers). */
int b2_quant_linear_gather(int kind, const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int block,
                           const void* w, int64_t ldw, int64_t N, const float* w_scale, int64_t w_scale_count,
                           const void* bias, int bias_dtype, int epilogue, int out_dtype, int64_t ldc,
                           int64_t col0, int world, int rank, void* const* outs, void* const* states,
                           uint32_t epoch, void* workspace, size_t workspace_bytes, void* stream);

/* The same column-parallel linear with the transfer on the copy engines:
 * the linear runs in `chunks` M-chunks (whole 256-row tiles, 1..8) on
 * `stream`, each chunk's block going to every peer's output by one 2-D
 * copy-engine copy on a per-peer copy stream while the next chunk is
 * multiplied; when a peer's copies are done a one-thread kernel on the same
 * copy stream adds 1 (release, system scope) to this rank's count in that
 * peer's state, and `stream` joins the copy streams.  The caller then enqueues
 * b2_gather_wait_ce, which advances this rank's sequence number and waits
 * (bounded, 2 s, status 0x107) until every peer's count reaches it.  No
 * per-call value: a step can be captured in a CUDA graph.  Same arguments and
 * requirements as b2_quant_linear_gather minus `epoch`; calls on one device
 * must not overlap (the copy streams and events are the library's, created
 * once per device). */
int b2_quant_linear_gather_ce(int kind, const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int block,
                              const void* w, int64_t ldw, int64_t N, const float* w_scale, int64_t w_scale_count,
                              const void* bias, int bias_dtype, int epilogue, int out_dtype, int64_t ldc,
                              int64_t col0, int world, int rank, void* const* outs, void* const* states, int chunks,
                              void* workspace, size_t workspace_bytes, void* stream);
int b2_gather_wait_ce(void* state, int world, int rank, void* stream);

/* Column-parallel INT8 activation exchange for stacks of column-parallel
 * linears (each layer's next layer reads whole rows of its output).  Rank
 * `rank` of `world` holds a column slice y [M, Ns] (16-byte aligned rows of
 * fp16/bf16/fp32, row stride ldy; Ns % 64 == 0, Ns <= 24576, Ns % block == 0,
 * Ns may be 0) of the layer output; block is the next layer's rotation
 * block (0/1 none, else a power of two <= 2048).
 *
 * Phase 1, b2_shard_amax: rotates the slice's blocks exactly as the
 * activation prologue does, reduces each row to the absmax of its rotated
 * values and stores it into slot [rank * M + row] of every rank's exchange
 * buffer xchg[q] (fp32 [world][M]); then releases `epoch` into slot `rank`
 * of every rank's state states[q] (b2_gather_state_bytes, 256-byte aligned).
 * Phase 2, b2_shard_codes, after b2_gather_wait(phase-1 state, epoch): the
 * row scale is max over the world slots of this rank's exchange buffer
 * (= the whole row's absmax; max is exact) / 127 (int8, quant 0) or / 448
 * (e4m3, quant 1); the slice's codes are written into columns [col0, col0 +
 * Ns) of every rank's code buffer q_outs[q] (row stride ldq bytes, ldq % 16
 * == 0, col0 % 16 == 0) and the scales into this rank's scale[M]; then
 * `epoch` is released into slot `rank` of every rank's (phase-2) state.
 * After b2_gather_wait on the phase-2 state every rank holds the codes and
 * scales that b2_act_quant computes on the whole row, bit for bit.  Each
 * phase needs its own state (epochs increase per state).  M == 0 launches
 * nothing and releases nothing.  No reference counterpart: the reference is
 * single-GPU; this is the multi-GPU form of its per-layer activation
 * quantization (production/MOSS_RDNA2_INT8/backend.py:112-127). */
int b2_shard_amax(const void* y, int y_dtype, int64_t M, int64_t Ns, int64_t ldy, int block, int world,
                  int rank, void* const* xchg, void* const* states, uint32_t epoch, void* stream);
int b2_shard_codes(const void* y, int y_dtype, int64_t M, int64_t Ns, int64_t ldy, int block, int quant,
                   int world, int rank, const void* xchg_local, void* const* q_outs, int64_t ldq, int64_t col0,
                   float* scale, void* const* states, uint32_t epoch, void* stream);

/* b2_shard_amax, b2_gather_wait on the phase-1 state and b2_shard_codes in
 * one cooperative launch: every CTA of the grid is resident, runs the
 * absmax pass, signals, waits (bounded, 2 s) for every rank's absmax slots
 * of epoch_amax, then runs the codes pass and releases epoch_codes into
 * every rank's phase-2 state.  Same arguments and results as the three
 * calls (xchg holds every rank's exchange buffer; this rank's own is
 * xchg[rank]); wait with b2_gather_wait on the phase-2 state.  A slice with
 * Ns == 0 runs the three calls.  Only one rank per GPU: ranks sharing a
 * device would wait on one another inside their kernels.  No reference
 * counterpart. */
int b2_shard_exchange(const void* y, int y_dtype, int64_t M, int64_t Ns, int64_t ldy, int block, int quant,
                      int world, int rank, void* const* xchg, void* const* amax_states, uint32_t epoch_amax,
                      void* const* q_outs, int64_t ldq, int64_t col0, float* scale, void* const* code_states,
                      uint32_t epoch_codes, void* stream);

/* Copy-engine copy of `rows` rows of `width_bytes` bytes between two device
 * buffers that may live on different GPUs (an IPC-mapped peer pointer, for
 * instance): the copy-engine counterpart of the gather, used to measure the
 * link bandwidth the fused gather is held against.  Asynchronous on `stream`. */
int b2_peer_copy_2d(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width_bytes, int64_t rows,
                    void* stream);

/* Enqueue a wait (one small kernel) until every one of the `world` slots of
 * the LOCAL gather state holds `epoch` or later, i.e. every rank's shard of
 * that call has landed in the local output buffer.  Bounded: after 2 s the
 * kernel gives up and sets b2_device_status to 0x107. */
int b2_gather_wait(const void* state, int world, uint32_t epoch, void* stream);

/* The gathered GEMM on operands already quantized (b2_qgemm's arguments:
 * codes a [M,K] with per-row a_scale, w [N,K] with w_scale; kind 0 INT8 or
 * 1 e4m3) with b2_quant_linear_gather's output contract: this rank's N
 * columns land at col0 of every rank's outs[q] and `epoch` is released into
 * slot `rank` of every rank's states[q]; wait with b2_gather_wait.  For
 * stacks whose layer inputs arrive as codes (b2_shard_codes).  No reference
 * counterpart (the reference is single-GPU). */
int b2_qgemm_gather(int kind, const void* a, int64_t lda, const float* a_scale, const void* w, int64_t ldw,
                    int64_t M, int64_t N, int64_t K, const float* w_scale, int64_t w_scale_count, const void* bias,
                    int bias_dtype, int epilogue, int out_dtype, int64_t ldc, int64_t col0, int world, int rank,
                    void* const* outs, void* const* states, uint32_t epoch, void* stream);

/* Allocation-free fused quantized linear: the same computation and results
 * as b2_quant_linear, for callers that cannot provide a workspace (a host
 * whose device memory is all owned by another allocator, a plugin calling
 * convention that carries only inputs and outputs, or code that must not call
 * cudaMalloc because it can synchronize the device).  The staging buffer is a
 * fixed device array inside the library: every GPU that loads the library
 * holds b2_quant_linear_noalloc_max_bytes() bytes for it until exit, a call
 * needing more staging (b2_quant_linear_workspace_bytes(M, K)) is rejected
 * with cudaErrorInvalidValue, and calls that overlap on the GPU share the
 * array and race -- keep them on one stream.  The first call on a device looks
 * up the array's address; make it before any stream capture.  Allocates
 * nothing.  No counterpart in the reference (its operators always allocate
 * their outputs through PyTorch). */
size_t b2_quant_linear_noalloc_max_bytes(void);
int b2_quant_linear_noalloc(int kind, const void* x, int x_dtype, int64_t M, int64_t K,
                            int64_t ldx, int block, const void* w, int64_t ldw, int64_t N,
                            const float* w_scale, int64_t w_scale_count, const void* bias,
                            int bias_dtype, int epilogue, void* out, int out_dtype, int64_t ldc,
                            void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B2_QLINEAR_H_ */
