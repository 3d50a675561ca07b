/*
 * mica_w8a8.h -- C ABI of libmica_w8a8.so, the B200 (sm_100a) W8A8 linear-layer hot path.
 *
 * Every entry point takes plain device pointers, element strides and sizes, plus a
 * cudaStream_t passed as void*. Nothing here allocates device memory, synchronises the
 * stream or aborts: each call returns an int status (MICA_OK == 0) and enqueues its
 * kernels on `stream`, so all of them can be captured into a CUDA graph (the fused
 * SwiGLU chain uses a cooperative launch, which graphs also accept).
 *
 * The reference serves this path through Python ctypes calls into AOT-compiled Triton
 * cubins (v0.5/serving/lib/int8_kernels.py) and torch fallbacks (lib/int8_quant.py).
 * Each entry point names the reference interface it replaces.
 *
 * Layouts (all row-major, last dimension contiguous):
 *   activations x   [M, K]  bf16 / fp16 / fp32, row stride ldx elements
 *   codes       q   [M, K]  int8,               row stride ldq bytes
 *   token scale s   [M]     fp32   (s = max(absmax_row, 1e-8) / 127)
 *   weights     W   [N, K]  int8,  K contiguous (the reference's qweight)
 *   channel sc. sw  [N]     fp32   (the reference's wscale)
 *   output      C   [M, N]  bf16 / fp16 / fp32, row stride ldc elements
 *
 * Alignment rules (checked; violations return MICA_ERR_ALIGN): every base pointer is
 * 16-byte aligned, every row stride in bytes is a multiple of 16.
 */
#ifndef MICA_W8A8_H
#define MICA_W8A8_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (never abort; 0 = success) -------------------------------------- */
#define MICA_OK               0
#define MICA_ERR_ARG          1   /* null pointer, bad dtype or flag                    */
#define MICA_ERR_SHAPE        2   /* M/N/K outside the supported range                  */
#define MICA_ERR_ALIGN        3   /* pointer or stride not 16-byte aligned              */
#define MICA_ERR_ARCH         4   /* current device is not sm_100                       */
#define MICA_ERR_CUDA         5   /* a CUDA runtime call failed (see mica_last_cuda_error) */
#define MICA_ERR_RANGE        6   /* a size exceeds int32 indexing                      */
#define MICA_ERR_WORKSPACE    7   /* workspace too small                                */
#define MICA_ERR_UNSUPPORTED  8   /* valid request this build does not implement        */

/* ---- element types ----------------------------------------------------------------- */
#define MICA_DT_BF16  0
#define MICA_DT_FP16  1
#define MICA_DT_FP32  2

/* ---- rounding of activation codes ---------------------------------------------------
 * HALF_AWAY: q = trunc(fl(v + 0.5)) for v >= 0, trunc(fl(v - 0.5)) otherwise, the
 *            reference GPU kernel (v0.5/serving/kernel_src/kernels.py:34-35).
 * HALF_EVEN: q = rint(v), the reference torch path torch.round
 *            (v0.5/serving/lib/int8_quant.py:70).                                       */
#define MICA_ROUND_HALF_AWAY  0
#define MICA_ROUND_HALF_EVEN  1

/* ---- RMSNorm conventions -------------------------------------------------------------
 * OFFSET: y = cast( (x * r) * (1 + w) ), one rounding, fp32 math
 *         (v0.5/serving/lib/fused_kernels.py:34 and the CPU branch :51-56).
 * WEIGHT: y = cast( w * cast(x * r) ), HF Qwen3RMSNorm (weight applied after the cast).
 * r = rsqrt(mean(x^2) + eps).                                                           */
#define MICA_NORM_OFFSET  0
#define MICA_NORM_WEIGHT  1

/* ---- device-side error word ---------------------------------------------------------
 * Kernels never trap. A bounded wait that runs out records one of these codes in a
 * per-device error word and the kernel returns early (its outputs are then invalid).  */
#define MICA_DEV_OK                 0
#define MICA_DEV_TIMEOUT_PRODUCER   1
#define MICA_DEV_TIMEOUT_MMA        2
#define MICA_DEV_TIMEOUT_EPILOGUE   3
#define MICA_DEV_TIMEOUT_GRID       4
#define MICA_DEV_TIMEOUT_DRAIN      5
#define MICA_DEV_TIMEOUT_SELFTEST   6
#define MICA_DEV_TIMEOUT_STREAMK    7   /* a stream-K CTA waited too long for its neighbour's partial */
#define MICA_DEV_BAD_LAUNCH         8   /* a kernel found its grid smaller than it needs and did nothing */

typedef struct mica_caps {
    int device;             /* CUDA ordinal queried                                     */
    int cc_major, cc_minor; /* compute capability                                       */
    int sm_count;           /* multiprocessors                                          */
    int supported;          /* 1 when this library's kernels run on the device          */
    int max_smem_optin;     /* bytes of opt-in shared memory per block                  */
    int abi_version;        /* MICA_ABI_VERSION                                         */
    int pair_clusters;      /* co-resident CTA pairs for the 256-row GEMM tiles         */
} mica_caps;

#define MICA_ABI_VERSION 5

/* Capability query. Replaces int8_kernels.available() (v0.5/serving/lib/int8_kernels.py:146-159)
 * and the capability probe in _device_cc (:130-143). Fills *caps for `device`.         */
int mica_query(int device, mica_caps* caps);

/* Loads every kernel of the library on the current device and sets its shared-memory
 * attributes, so the first real call does no lazy set-up (and may be graph-captured).
 * Replaces int8_kernels.preload() (v0.5/serving/lib/int8_kernels.py:217-224).
 * Returns MICA_OK and writes the number of kernels prepared to *n_kernels (may be NULL). */
int mica_preload(int* n_kernels);

/* Text of the last CUDA runtime error seen by this thread's calls (empty if none).      */
const char* mica_last_cuda_error(void);

/* Reads the current device's error word into *code and clears it. Synchronises
 * `stream` (diagnostics only, never on the hot path).                                   */
int mica_device_error(int* code, void* stream);

/* Per-token int8 activation quantiser: optional smoothing multiply x*inv[k], absmax,
 * s = max(absmax, 1e-8)/127, q = round(x/s) clamped to [-127, 127].
 * Replaces int8_kernels.act_quant (v0.5/serving/lib/int8_kernels.py:325-353) launching
 * the Triton act_quant (v0.5/serving/kernel_src/kernels.py:15-38), and the torch
 * fallback int8_quant.quant_act (v0.5/serving/lib/int8_quant.py:64-74).
 * x_dtype: MICA_DT_*. inv may be NULL. M >= 0, 1 <= K, K % 8 == 0.                     */
int mica_act_quant(const void* x, int x_dtype, long ldx, const float* inv,
                   int8_t* q, long ldq, float* s, int M, int K, int round_mode,
                   void* stream);

/* Fused RMSNorm + per-token quantiser (the prologue of every QLinear that follows a norm).
 *   sum  = residual ? x + residual (rounded to x dtype) : x
 *   y    = RMSNorm(sum) with gamma in the x dtype, norm_style MICA_NORM_*
 *   q, s = per-token quantisation of y (as mica_act_quant, with optional inv)
 * Optional outputs: y_out (normalised activations, x dtype, row stride ldy) and
 * sum_out (the residual-added stream, x dtype, row stride ldsum); either may be NULL.
 * q and s may both be NULL for a norm-only call (then y_out is required).
 * Replaces fused_kernels.rms_norm (v0.5/serving/lib/fused_kernels.py:50-83, kernel :11-35)
 * followed by int8_kernels.act_quant.  x_dtype: MICA_DT_BF16 or MICA_DT_FP16.            */
int mica_rmsnorm_quant(const void* x, int x_dtype, long ldx,
                       const void* residual, long ldr,
                       const void* gamma, int norm_style, float eps,
                       const float* inv,
                       void* y_out, long ldy, void* sum_out, long ldsum,
                       int8_t* q, long ldq, float* s,
                       int M, int K, int round_mode, void* stream);

/* W8A8 GEMM on tcgen05 tensor cores (kind::i8, int32 accumulation in tensor memory):
 *   C[m, n] = cast( ((float)acc[m, n] * sa[m]) * sb[n]  (+ bias[n]) ),
 *   acc[m, n] = sum_k A[m, k] * B[n, k]       (exact int32)
 * No fused multiply-add in the epilogue; the cast is round-to-nearest-even.
 * bias may be NULL. c_dtype: MICA_DT_*.  1 <= M, N; K % 16 == 0.
 * Replaces int8_kernels.mm_i8 (v0.5/serving/lib/int8_kernels.py:359-406) launching the
 * Triton mm_i8 (v0.5/serving/kernel_src/kernels.py:41-69), and the torch fallback
 * torch_int_mm + dequant (v0.5/serving/lib/int8_runtime.py:186-192).                   */
int mica_w8a8_gemm(const int8_t* A, long lda, const int8_t* B, long ldb,
                   const float* sa, const float* sb, const float* bias,
                   void* C, int c_dtype, long ldc,
                   int M, int N, int K, void* stream);

/* As mica_w8a8_gemm with an explicit output tile, used by the tile tuner:
 *   block_m 128 = one CTA per tile; 256 = a pair of CTAs on two SMs sharing each MMA
 *           (tcgen05 cta_group::2), 0 = library choice;
 *   block_n 64 / 128 / 256 (pairs: 128 / 256), 0 = library choice; 320 (single CTAs, splits
 *           0 or 1) is for grids that fit one wave at that width (MICA_ERR_UNSUPPORTED otherwise):
 *           the library picks it when 128 x 256 tiles would need between one and two waves;
 *   max_ctas caps the persistent grid (0 = all SMs / all co-resident pairs);
 *   splits   K split of each 128-row tile across a cluster of that many CTAs, reduced in
 *           distributed shared memory (exact): 0 = library choice (split only when fewer
 *           than half the SMs would get a tile), 1 = never, 2..8 = forced (MICA_ERR_UNSUPPORTED
 *           when a rank would get no k-block). Ignored with max_ctas > 0; not with block_m 256.
 *           MICA_SPLIT_STREAM_K asks for the stream-K kernel, which needs a workspace: use
 *           mica_w8a8_gemm_ex (here it returns MICA_ERR_WORKSPACE).                          */
#define MICA_SPLIT_STREAM_K (-1)
int mica_w8a8_gemm_cfg(const int8_t* A, long lda, const int8_t* B, long ldb,
                       const float* sa, const float* sb, const float* bias,
                       void* C, int c_dtype, long ldc,
                       int M, int N, int K, int block_m, int block_n, int max_ctas, int splits,
                       void* stream);

/* As mica_w8a8_gemm_cfg with a device workspace, which lets the library run a grid whose
 * last wave would leave most SMs idle as stream-K: one CTA per SM, every CTA the same number
 * of (tile, k-block) units, a tile cut between two CTAs finished by the one that reaches it
 * last from the other's int32 partial (exact: the same int32 sums as the data-parallel
 * kernel). Used by the library choice (splits 0, block_m 128 or 0, max_ctas 0) when it
 * shortens the critical path, and by splits = MICA_SPLIT_STREAM_K (block_n 128 or 256).
 * workspace: mica_w8a8_gemm_workspace_bytes(...) bytes for the same arguments, 16-byte
 * aligned, reserved for this call until it completes on `stream` (the call clears what it
 * needs). With splits 0 and a NULL or smaller workspace the data-parallel kernel runs.
 * The library choice uses it where 128 x 320 tiles cannot fit the grid in one wave (e.g. M
 * 2048, N 3072, K 9728). No counterpart in the reference (its Triton mm_i8 grid is one
 * program per tile, v0.5/serving/kernel_src/kernels.py:41-69).                            */
int mica_w8a8_gemm_ex(const int8_t* A, long lda, const int8_t* B, long ldb,
                      const float* sa, const float* sb, const float* bias,
                      void* C, int c_dtype, long ldc,
                      int M, int N, int K, int block_m, int block_n, int max_ctas, int splits,
                      void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes mica_w8a8_gemm_ex uses with these arguments on the current device
 * (0: none; also 0 for arguments it would reject).                                      */
size_t mica_w8a8_gemm_workspace_bytes(int M, int N, int K, int block_m, int block_n, int max_ctas, int splits);

/* Fused MLP front half: gate_up W8A8 GEMM + SwiGLU + next-layer per-token quantisation.
 *   Bgu [2*I, K]: gate and up weight rows interleaved in groups of 16
 *        (rows 32j..32j+15 = gate rows 16j..16j+15, rows 32j+16..32j+31 = up rows
 *         16j..16j+15); sgu, bias_gu follow the same order (bias_gu may be NULL).
 *   g = bf16(deq(gate)), u = bf16(deq(up)),  h = bf16( bf16(silu(g)) * u )  -> h_out [M, I]
 *   then q_out / s_out = per-token int8 quantisation of h * inv_h (round_mode as above);
 *   inv_h [I] is down_proj's inv_smooth, or NULL (v0.5/serving/lib/int8_quant.py:64-67).
 * gate_proj and up_proj must share their input quantisation (no smoothing, or the same
 * inv_smooth, applied by the caller's act_quant / rmsnorm_quant); with different smoothing
 * use two mica_w8a8_gemm calls and mica_swiglu_quant.
 * Replaces gate_proj + up_proj QLinears, fused_kernels.swi_glu
 * (v0.5/serving/lib/fused_kernels.py:85-96, kernel :37-44) and the act_quant of
 * down_proj's input (v0.5/serving/lib/fast_runtime.py:126-132).
 * workspace: at least mica_swiglu_workspace_bytes(M) bytes, 16-byte aligned.
 * I % 16 == 0, K % 16 == 0.                                                             */
size_t mica_swiglu_workspace_bytes(int M);
int mica_w8a8_gemm_swiglu_quant(const int8_t* A, long lda, const int8_t* Bgu, long ldb,
                                const float* sa, const float* sgu, const float* bias_gu,
                                const float* inv_h,
                                void* h_out, long ldh,
                                int8_t* q_out, long ldq, float* s_out,
                                int M, int I, int K, int round_mode,
                                void* workspace, size_t workspace_bytes, void* stream);

/* The same fused gate_up + SwiGLU + requantisation, for callers that cannot allocate
 * device memory. No counterpart in the reference.
 * Who needs it: a host that has already handed all of the GPU's memory to its own
 * planner (a serving runtime that sizes its context cap against the whole device), or a
 * plugin whose host owns the allocator and forbids cudaMalloc on the serving path because
 * an allocation there can block or fail in the middle of a request. Such callers cannot
 * supply the workspace that mica_w8a8_gemm_swiglu_quant needs.
 * Instead, this entry point uses a scratch array compiled into the library
 * (MICA_NOALLOC_SCRATCH_BYTES per GPU that loads it, held until the process exits). It
 * calls no cudaMalloc, cudaFree or other allocating routine. The caller still passes every
 * input and output.
 * Limit: M <= MICA_NOALLOC_MAX_ROWS; larger M returns MICA_ERR_WORKSPACE before any work.
 * Set-up: the first call on each device looks up the scratch array's device address,
 * with that device current. Make that first call before any stream capture (a warm-up
 * call is enough).
 * Sharing: every call on a device uses the same scratch, and each call clears what must
 * start at zero. Calls whose kernels overlap on the GPU (other streams, other threads)
 * race on that scratch: serialise them.                                                   */
#define MICA_NOALLOC_MAX_ROWS       65536
#define MICA_NOALLOC_SCRATCH_BYTES  (65536 * 4 + 16)
int mica_w8a8_gemm_swiglu_quant_noalloc(const int8_t* A, long lda, const int8_t* Bgu, long ldb,
                                        const float* sa, const float* sgu, const float* bias_gu,
                                        const float* inv_h,
                                        void* h_out, long ldh,
                                        int8_t* q_out, long ldq, float* s_out,
                                        int M, int I, int K, int round_mode, void* stream);

/* SwiGLU of two projection outputs, then down_proj's per-token quantisation:
 *   h = bf16( bf16(silu(g)) * u )  -> h_out [M, I] (optional),
 *   q / s = per-token int8 quantisation of h * inv (inv [I] optional; q and s together,
 *           optional; at least one of h_out and q).
 * For MLPs whose gate_proj and up_proj have different smoothing (two quantisations of the
 * same input, so no shared GEMM operand). Replaces fused_kernels.swi_glu
 * (v0.5/serving/lib/fused_kernels.py:85-96, kernel :37-44) and the act_quant that
 * down_proj's QLinear runs on its output (v0.5/serving/lib/int8_runtime.py:181-182).
 * g, u: dtype MICA_DT_BF16 / MICA_DT_FP16 [M, I] with row strides ldg, ldu; I % 8 == 0.   */
int mica_swiglu_quant(const void* g, long ldg, const void* u, long ldu, int dtype, const float* inv,
                      void* h_out, long ldh, int8_t* q, long ldq, float* s,
                      int M, int I, int round_mode, void* stream);

/* Option-logit scorer for the last position of each request:
 *   hn[b]       = optional RMSNorm of h[b] (gamma NULL = h used as given; gamma has
 *                 h's dtype, norm_style MICA_NORM_*)
 *   logits[b,r] = sum_d float(hn[b,d]) * rows[r,d]        (fp32, rows = gathered lm_head)
 *   probs[b, lo_b..hi_b) = softmax(logits[b, lo_b..hi_b)), other entries 0.
 * lo/hi may be NULL (softmax over all n_rows). probs may be NULL (logits only).
 * Replaces the readout closure (v0.5/serving/lib/release_runtime.py:302-306) and the
 * slice + softmax (v0.5/serving/lib/release_runtime.py:430-431, :509-522).
 * h_dtype: MICA_DT_BF16/FP16/FP32. D % 8 == 0, 1 <= n_rows <= 4096.                    */
int mica_option_logits(const void* h, int h_dtype, long ldh,
                       const void* gamma, int norm_style, float eps,
                       const float* rows, int n_rows, int D,
                       const int* lo, const int* hi,
                       float* logits, float* probs, int B, void* stream);

/* Per-head RMSNorm of q and k followed by the rotary embedding, in place on the QKV GEMM
 * output (bf16 rows [q: H*D | k: KV*D | v], row stride ld elements). Reproduces HF Qwen3's
 * bf16 sequence: y = w * bf16(x * rsqrt(mean(x^2) + eps)), then
 * bf16(bf16(y * cos) + bf16(rotate_half(y) * sin)). cos/sin: bf16 [positions, D];
 * pos: int64 [S] token positions on the device, or NULL for pos0 + row index.
 * D in {64, 128}. Replaces the q_norm / k_norm / apply_rotary_pos_emb torch ops around the
 * QKV projection (the reference runs them in torch, v0.5/serving/lib/prefill_engine.py:308-324). */
int mica_qk_norm_rope(void* qkv, long ld, const void* q_w, const void* k_w, const void* cos, const void* sin,
                      const int64_t* pos, long pos0, int S, int H, int KV, int D, float eps, void* stream);

/* Causal grouped-query attention forward of the prefill on tcgen05 tensor cores, reading Q, K
 * and V in place from the QKV projection's output:
 *   qkv [B * L, >= (H + 2 KV) * D] bf16, row stride ld_qkv elements: per row q (H heads of D),
 *       then k (KV heads), then v (KV heads); rows b * L .. b * L + L - 1 are request b;
 *   out [B * L, >= H * D] bf16, row stride ld_out: out[t, h] = sum over keys s <= t of request
 *       b of softmax_s(scale * q[t, h] . k[s, h / (H / KV)]) v[s, h / (H / KV)].
 * fp32 scores and accumulation. D == 128, H % KV == 0. Replaces the torch SDPA call of the
 * reference's prefill (v0.5/serving/lib/prefill_engine.py:308-324, lib/fast_runtime.py:189-220;
 * the reference's own Triton kernel is v0.5/serving/kernel_src/kernels.py:72-124).           */
int mica_attention_prefill(const void* qkv, long ld_qkv, void* out, long ld_out, int B, int L, int H, int KV, int D,
                           float scale, void* stream);

/* Failure-detection self-test: launches one block that waits on a barrier nothing
 * ever arrives on, with a wait limit of limit_us microseconds. The kernel gives up,
 * records MICA_DEV_TIMEOUT_SELFTEST in *status_dev (device int) and returns; the GPU
 * context stays usable. No counterpart in the reference (its start-up self-test,
 * v0.5/serving/lib/int8_runtime.py:362-443, only bounds a child process on the host). */
int mica_selftest_wait_timeout(int* status_dev, int limit_us, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MICA_W8A8_H */
