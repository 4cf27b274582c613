/*
 * nf4b200.h - C ABI of the B200 (sm_100a) NF4 hot-path library (libnf4b200.so).
 *
 * The reference (bitNtech/ttspipe) reaches its kernels through Python ctypes
 * and the CUDA driver API (app/engine/nvrtc.py:184-199). This library replaces
 * those NVRTC-compiled kernels with nvcc-built sm_100a ones behind plain C
 * entry points: pointers and sizes only, no torch types, no exceptions.
 *
 * Conventions shared by every entry point:
 *   - All tensor pointers are device pointers, contiguous, row-major.
 *   - Activations are bf16 (uint16 bit patterns) unless an _ex call or
 *     nf4b_gemm_opts.dtype selects fp16; accumulation is fp32.
 *   - Alignment is checked on the host (NF4B_ERR_ALIGN, nothing launched):
 *     packed weights and matmul inputs 16 bytes, workspaces 256 bytes, other
 *     bf16/fp16 arrays 2 bytes, fp32 rotary tables 4, int64 values 8; each
 *     entry point notes any stricter rule.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). Nothing here
 *     synchronises the host or allocates device memory, so every call can be
 *     captured into a CUDA graph.
 *   - Return 0 on success or a negative NF4B_ERR_* code; the message of the
 *     last failure on the calling thread is nf4b_last_error().
 */
#ifndef NF4B200_H
#define NF4B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. Argument errors are detected on the host before any launch. */
#define NF4B_OK 0
#define NF4B_ERR_ARG (-1)         /* null pointer or out-of-range scalar      */
#define NF4B_ERR_SHAPE (-2)       /* shape the kernels do not serve           */
#define NF4B_ERR_ALIGN (-3)       /* pointer not aligned as required          */
#define NF4B_ERR_DTYPE (-4)       /* dtype the kernels do not serve           */
#define NF4B_ERR_WORKSPACE (-5)   /* workspace missing or too small           */
#define NF4B_ERR_LAUNCH (-6)      /* CUDA launch / runtime error              */
#define NF4B_ERR_DEVICE (-7)      /* current device is not sm_100             */

/* Epilogues fused into the matmul's store (app/engine/nf4gemv.py:424). */
#define NF4B_EPI_NONE 0
#define NF4B_EPI_RESIDUAL 1   /* y = operand + x W^T                          */
#define NF4B_EPI_SILU_GATE 2  /* y = silu(operand) * x W^T                    */

/* Element types of the rotary table (app/engine/fusedops.py:96-101). */
#define NF4B_F32 0
#define NF4B_F16 1
#define NF4B_BF16 2

/*
 * One bitsandbytes NF4 weight, read in place (app/engine/nf4gemv.py:343-377
 * lists the QuantState fields the reference reads).
 *   packed      uint8 [n_out, k_in/2]; byte j = (q[2j] << 4) | q[2j+1]
 *   nested = 0: absmax fp32 [n_out * k_in / blocksize]; absmax_code, code2 unused
 *   nested = 1: absmax_code uint8 [n_out * k_in / blocksize] (QuantState.absmax),
 *               absmax fp32 [ceil(nblocks / blocksize2)] (state2.absmax),
 *               code2 fp32 [256] (state2.code), offset (QuantState.offset);
 *               scale[b] = code2[absmax_code[b]] * absmax[b / blocksize2] + offset
 *   blocksize, blocksize2: powers of two; blocksize >= 64; k_in % blocksize == 0
 */
typedef struct nf4b_weight {
  const uint8_t* packed;
  const uint8_t* absmax_code;
  const float* absmax;
  const float* code2;
  float offset;
  int32_t n_out;
  int32_t k_in;
  int32_t blocksize;
  int32_t blocksize2;
  int32_t nested;
} nf4b_weight;

/* Library version (major * 10000 + minor * 100 + patch). */
int nf4b_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* nf4b_last_error(void);

/*
 * The library's device error word: non-zero after a kernel gave up on a
 * bounded wait (a pipeline barrier that never completed): bit 0 the GEMM,
 * bit 1 the GEMV, bit 2 decode attention's KV copies, bit 3 a decode step's
 * handoff. Synchronises the device to read it; `clear`
 * resets it; -1 if it cannot be read. The outputs of a call that set it are
 * invalid. The abort paths still count every CTA / warp into the workspace
 * counters (so the last arriver returns them to zero) and the decode step takes
 * a new flag space per launch; a caller that wants certainty zeroes a workspace
 * again after a non-zero word before reusing it. No counterpart in the
 * reference, whose kernels have no waits.
 */
int nf4b_device_error(int clear);

/*
 * Y[rows, n_out] = epi(X[rows, k_in] . dequant(W)^T).
 * Replaces the `nf4_mma` launch of nf4gemv.matmul (app/engine/nf4gemv.py:427-479):
 * 1..8 rows (decode and batched decode) run the streaming GEMV - the
 * register-fed kernel for blocksize-64 weights with k_in % 256 == 0, which
 * decodes each weight once for all rows - and larger row counts the tcgen05
 * GEMM. `operand` has Y's shape (epi != NONE).
 * `workspace` must hold nf4b_gemm_workspace_size(w, rows) bytes and be zeroed
 * once before its first use; every call leaves it zeroed again. One workspace
 * per stream: calls that overlap on the GPU must not share one. For the GEMM
 * the workspace holds split-K partial sums (the k range is split across CTAs
 * when the output tiles alone cannot fill the GPU, and each tile's last CTA
 * sums the splits in order); a GEMM given no (or too small a) workspace runs
 * unsplit, with the same results up to fp32 summation order.
 */
int nf4b_gemm(const nf4b_weight* w, const void* x, void* y, int rows, int epi,
              const void* operand, void* workspace, size_t workspace_bytes, void* stream);

/* Options of nf4b_gemm_ex. No counterpart in the reference. */
typedef struct nf4b_gemm_opts {
  /* Weights a LATER call on this stream will read, or NULL. Their packed
   * codes and first-level scales are streamed into L2 by the GEMV's warps
   * while it runs, so those launches find their weights in L2 instead of
   * waiting on HBM. Purely a hint: results do not depend on it. */
  const nf4b_weight* prefetch_next;
  const nf4b_weight* prefetch_next2;
  /* Non-NULL: x is first RMS-normalised with this bf16 [k_in] weight and
   * norm_eps inside the launch, with exactly the arithmetic of nf4b_rms_norm,
   * and the matmul reads the normalised x (it is never written out): the
   * reference's attention_norm / ffn_norm before wqkv / w1,w3 as one launch.
   * Served when x fits the decode GEMV's shared-memory staging: the
   * register-fed kernel's (1..8 rows, blocksize 64, k_in % 256 == 0,
   * rows * k_in * 2 <= 162 KB), else the pair kernel's (1..4 rows,
   * k_in % 128 == 0, rows * k_in * 2 <= 40 KB); NF4B_ERR_SHAPE otherwise. */
  const void* norm_weight;
  float norm_eps;
  /* Activation type of x, operand, y and norm_weight: 0 or NF4B_BF16 = bf16,
   * NF4B_F16 = fp16 (the reference's own kernel serves fp16 only,
   * app/engine/nf4gemv.py:439; its TTS_HALF default, app/config.py:107). fp16
   * runs the register-fed decode GEMV for 1..8 rows (blocksize 64,
   * k_in % 256 == 0, 32-byte aligned packed codes; a fused RMSNorm and the
   * gated pair as for bf16) and the tcgen05 GEMM for every other row count,
   * with the reference's rounding points in fp16 (fp32 accumulation; the
   * matmul output and each epilogue op rounded to fp16). The fused rotary
   * store and the chain / decode-step launches are bf16 only. Any other value:
   * NF4B_ERR_DTYPE. */
  int dtype;
} nf4b_gemm_opts;

/* nf4b_gemm with options (opts may be NULL). */
int nf4b_gemm_ex(const nf4b_weight* w, const void* x, void* y, int rows, int epi,
                 const void* operand, void* workspace, size_t workspace_bytes,
                 const nf4b_gemm_opts* opts, void* stream);

/*
 * The wqkv projection of one token with the rotary + KV-cache write fused into
 * its store (qk_rope_kv without q/k norm, app/engine/fusedlayer.py:56-92):
 * y = x W^T (bf16, as nf4b_gemm), q heads rotated into q_out, k heads rotated
 * into k_cache row *pos, v heads copied into v_cache row *pos (a *pos outside
 * [0, max_len) writes no cache row) - bit-identical to nf4b_gemm followed by
 * nf4b_qk_rope_kv with no norm weights. Output features are n_head query
 * heads, then n_kv key heads, then n_kv value heads, 128 wide; freqs is this
 * token's rotary row (128 values, (cos, sin) pairs). Serves one row on the
 * register-fed decode GEMV (blocksize 64, k_in % 256 == 0, 32-byte aligned
 * packed weight); anything else returns NF4B_ERR_SHAPE (make the two calls).
 * opts as nf4b_gemm_ex (a fused RMSNorm of x is allowed).
 */
typedef struct nf4b_rope_kv {
  const void* freqs;
  int freqs_dtype; /* NF4B_F32 / NF4B_F16 / NF4B_BF16 */
  const int64_t* pos;
  void* q_out;     /* [n_head * 128] bf16 */
  void* k_cache;   /* (n_kv, max_len, 128) bf16 */
  void* v_cache;
  int n_head, n_kv, max_len;
} nf4b_rope_kv;

int nf4b_gemm_qkv_rope(const nf4b_weight* w, const void* x, void* y, const nf4b_rope_kv* rk, void* workspace,
                       size_t workspace_bytes, const nf4b_gemm_opts* opts, void* stream);

/*
 * The FeedForward gate of a W1/W3 pair sharing x in ONE launch:
 * y = bf16(bf16(silu(bf16(x W1^T))) * bf16(x W3^T)), the rounding points of the
 * fork's w2(F.silu(w1(x)) * w3(x)) (app/engine/fusedlayer.py:265-266, where it
 * is two nf4gemv.matmul launches, the second with EPI_SILU_GATE). x W1^T is
 * never written out. Serves 1..8 rows on the register-fed kernel (blocksize
 * 64, k_in % 256 == 0) and 1..4 rows with k_in % 128 == 0 otherwise
 * (NF4B_ERR_SHAPE beyond: the caller then issues the two matmuls; fp16: the
 * register-fed kernel only). w1 and w3 must agree in
 * shape and quantisation. Workspace as nf4b_gemm (nf4b_gemm_workspace_size of
 * w1 covers it). No reference counterpart as a single call.
 */
int nf4b_gemm_gated(const nf4b_weight* w1, const nf4b_weight* w3, const void* x, void* y, int rows,
                    void* workspace, size_t workspace_bytes, const nf4b_gemm_opts* opts, void* stream);

/* One job of nf4b_gemv_chain. */
typedef struct nf4b_chain_job {
  const nf4b_weight* w;     /* the weight; for a gated pair, W1                      */
  const nf4b_weight* w3;    /* gated pair: W3 (same shape and quantisation); else NULL */
  const void* x;            /* [rows, k_in] bf16, 16-byte aligned; may be an earlier job's y */
  void* y;                  /* [rows, n_out] bf16                                     */
  const void* operand;      /* epilogue operand [rows, n_out] bf16 (may be an earlier job's y), or NULL */
  int32_t epi;              /* NF4B_EPI_*; ignored for gated pairs                    */
  const void* norm_weight;  /* non-NULL: x is first RMS-normalised with this bf16 [k_in] weight, exactly
                               as nf4b_rms_norm (then the matmul reads the normalised x) */
  float norm_eps;
} nf4b_chain_job;

#define NF4B_MAX_CHAIN_JOBS 40

/*
 * Up to NF4B_MAX_CHAIN_JOBS decode GEMVs that depend on one another, in ONE
 * persistent launch: job j reads its x and operand only after every output of
 * jobs 0..j-1 is written, so a transformer block's matmul sequence
 * (wo + residual -> RMSNorm -> the W1/W3 gate -> w2 + residual, and so on) runs
 * without a launch between its steps. Each job computes what nf4b_gemm (or
 * nf4b_gemm_gated, after nf4b_rms_norm when norm_weight is given) computes,
 * within the GEMV's rounding. Serves 1..4 rows of blocksize-64 NF4 weights
 * with k_in % 256 == 0 and rows * k_in * 2 <= 40 KB (NF4B_ERR_SHAPE
 * otherwise). The workspace (nf4b_gemv_chain_workspace_size) is zeroed once
 * by the caller and left zeroed by every call. No reference counterpart: the
 * reference launches every matmul, norm and gate separately
 * (app/engine/fusedlayer.py:212-269).
 */
int nf4b_gemv_chain(const nf4b_chain_job* jobs, int n_jobs, int rows, void* workspace,
                    size_t workspace_bytes, void* stream);

size_t nf4b_gemv_chain_workspace_size(const nf4b_chain_job* jobs, int n_jobs, int rows);

#define NF4B_MAX_STEP_JOBS 152

/*
 * A whole decode step's dependent matmuls in ONE launch: up to
 * NF4B_MAX_STEP_JOBS jobs with nf4b_gemv_chain's semantics (job j reads its x
 * and operand only after every output of jobs 0..j-1 is written; x and
 * operand may be earlier jobs' y; a job's norm_weight RMS-normalises its x
 * first, exactly as nf4b_rms_norm), for 1 or 2 activation rows. It replaces
 * the sequence of nf4gemv.matmul launches the reference's decode_block issues
 * per block (app/engine/fusedlayer.py:212-269; the graph of them that
 * graphs.DecodeGraphs replays), e.g. 36 layers x (wqkv, wo + residual, the
 * W1/W3 gate, w2 + residual) = 144 jobs.
 * One CTA per SM (a cooperative launch) streams the weights of job j + 1
 * into registers while job j's outputs are handed over; a job whose x is the
 * previous job's y reads it from flag-tagged handoff words in the workspace
 * (one L2 round trip), any other boundary is a full barrier. Each job equals
 * nf4b_gemm (or nf4b_gemm_gated) up to fp32 summation order; results are
 * deterministic. Serves blocksize-64 weights with k_in % 256 == 0,
 * k_in <= 10240, n_out % 16 == 0, 32-byte aligned packed weights (NF4B_ERR_*
 * otherwise). A job whose x (or operand) is the previous job's y must match
 * its shape. The workspace (nf4b_decode_step_workspace_size) is zeroed once
 * before its first use; the step keeps a launch counter in it and must have
 * it to itself (one workspace per stream). No reference counterpart as a
 * single call.
 */
int nf4b_decode_step(const nf4b_chain_job* jobs, int n_jobs, int rows, void* workspace,
                     size_t workspace_bytes, void* stream);

size_t nf4b_decode_step_workspace_size(const nf4b_chain_job* jobs, int n_jobs, int rows);

/*
 * Test hook for failure detection (not for production use): nf4b_decode_step
 * whose waits give up after `wait_ns` nanoseconds, and whose boundary before
 * job `stall_job` (-1: none) waits for a flag that is never written, so that
 * boundary's wait runs out. The kernel then records bit 3 in
 * nf4b_device_error and returns; nothing faults, and the next launch on the
 * same workspace is unaffected.
 */
int nf4b_debug_decode_step(const nf4b_chain_job* jobs, int n_jobs, int rows, void* workspace,
                           size_t workspace_bytes, int stall_job, unsigned long long wait_ns, void* stream);

/*
 * Test hook for failure detection (not for production use), for the
 * tcgen05 GEMM (more than 8 rows) of the current device: every later GEMM
 * launch's waits give up after `wait_ns` nanoseconds, and with `skip_x0` = 1
 * its producer leaves the first k block's activation tile unrequested, so the
 * barrier that copy would complete never does and the waits on it run out.
 * The launch then records bit 0 in nf4b_device_error and returns (its outputs
 * are invalid); nothing faults. nf4b_debug_gemm_hook(0, 2000000000) restores
 * normal operation. No counterpart in the reference, whose kernels have no waits.
 */
int nf4b_debug_gemm_hook(int skip_x0, unsigned long long wait_ns);

/* Bytes of workspace nf4b_gemm needs for this weight and row count. */
size_t nf4b_gemm_workspace_size(const nf4b_weight* w, int rows);

/* Size of the device scratch compiled into the library for nf4b_gemm_noalloc. */
#define NF4B_NOALLOC_SCRATCH_BYTES (4u << 20)

/*
 * nf4b_gemm for callers that cannot allocate device memory (a real-time audio
 * callback that must not touch an allocator, a cgo/JNI host holding only raw
 * device pointers from another runtime, a graph being recorded): the GEMV's
 * partial sums and counters live in a 4 MiB scratch array built into the
 * library, which every GPU that loads it keeps until exit. No counterpart in
 * the reference. Limits: GEMV calls (1..8 rows) whose scratch need
 * (nf4b_gemm_workspace_size) exceeds NF4B_NOALLOC_SCRATCH_BYTES fail with
 * NF4B_ERR_WORKSPACE. More than 8 rows run the tensor-core GEMM, which puts
 * its split-K partial sums in the same scratch when they fit (so it splits
 * exactly as nf4b_gemm with a workspace does) and otherwise runs unsplit;
 * those calls share the scratch too. The first call on a device looks the
 * scratch's device address up and keeps it for the life of the process, so
 * make it before any stream capture, and do not reset the device
 * (cudaDeviceReset) between calls. All calls share the scratch: each clears
 * its counters first, and calls that overlap on the GPU (other streams or
 * threads) race.
 */
int nf4b_gemm_noalloc(const nf4b_weight* w, const void* x, void* y, int rows, int epi,
                      const void* operand, void* stream);

/*
 * y[n_out] = bf16(x W^T) for a dense bf16 weight W[n_out, k_in] (row-major)
 * and one activation row x[k_in], fp32 accumulation - the fork's bf16 output
 * heads (the slow AR's LM head, the fast AR's codebook heads), which the
 * reference runs through torch. k_in in {1024, 2048, 2560, 4096}; w and x
 * 16-byte aligned. A non-NULL bf16 `norm_weight` [k_in] RMS-normalises x first
 * (with norm_eps), exactly as nf4b_rms_norm, inside the launch: the final norm
 * before a head. No reference counterpart as a single call.
 */
int nf4b_dense_gemv(const void* w, const void* x, void* y, int n_out, int k_in, const void* norm_weight,
                    float norm_eps, void* stream);

/*
 * Draw one token id from a bf16 logit row, on the device (graph-capturable):
 * the fork's sampler as the reference calls it (app/engine/graphs.py:55-73;
 * fused in app/engine/fusedsample.py) - logits sorted descending, positions
 * past top_k (<= 64) or past cumulative softmax probability top_p (softmax of
 * the unscaled logits over the whole vocabulary) dropped except the first,
 * the kept logits divided by max(temperature, 1e-5), softmax, one draw. The
 * draw uses one uniform from a counter-based hash of (seed, *step) (step may
 * be NULL: 0), so a run is reproducible from its seed. Writes out[0] (int64).
 * vocab <= 262144. The workspace (nf4b_sample_workspace_size) is zeroed once
 * by the caller and left zeroed.
 */
int nf4b_sample(const void* logits, int vocab, float temperature, float top_p, int top_k,
                unsigned long long seed, const int64_t* step, int64_t* out, void* workspace,
                size_t workspace_bytes, void* stream);

size_t nf4b_sample_workspace_size(int vocab);

/*
 * Dual-AR frame bookkeeping on the device (graph-capturable; one small
 * launch each instead of the framework's compare / gather / copy kernels).
 * The token logic of the reference's decode step (app/engine/graphs.py:105-127).
 * Embedding tables are bf16 [rows, dim] with dim % 8 == 0, 16-byte aligned;
 * token ids are int64 and clamped to their table.
 *
 * nf4b_embed_rows: out row r = table row ids[r], r < n_ids.
 *
 * nf4b_frame_select: the repetition-aware choice of the semantic token and
 * the fast AR's first input. main' = *high when *main is a semantic id
 * (sem_begin <= *main < sem_begin + codebook_size) that occurs in
 * recent[0..n_recent), else *main; tokens[0] = main'; tokens[1] = a =
 * clamp(main' - sem_begin, 0, codebook_size - 1); h = fast_emb row a.
 *
 * nf4b_frame_advance: the next frame's input and counters. x = bf16(
 * float(sem_emb row tokens[0]) + s), s = the fp32 sum in codebook order of
 * float(cb_emb[i] row tokens[1 + i]) for i < n_codebooks (cb_emb is
 * [n_codebooks, codebook_size, dim]); recent <- [tokens[0], recent[0..n-2]];
 * *pos += 1; *step += 1. n_codebooks <= 32.
 */
int nf4b_embed_rows(const void* table, long long rows, const int64_t* ids, int n_ids, int dim, void* out,
                    void* stream);
int nf4b_frame_select(const int64_t* main_tok, const int64_t* high_tok, const int64_t* recent, int n_recent,
                      long long sem_begin, long long codebook_size, int64_t* tokens, const void* fast_emb, int dim,
                      void* h, void* stream);
int nf4b_frame_advance(const void* sem_emb, long long vocab, const void* cb_emb, long long codebook_size,
                       int n_codebooks, const int64_t* tokens, int dim, void* x, int64_t* recent, int n_recent,
                       int64_t* pos, int64_t* step, void* stream);

/*
 * out[n_out, k_in] = RNE_bf16(NF4[q] * scale) - bitsandbytes' dequantize_4bit
 * to bf16 (the per-element value of app/engine/nf4gemv.py:185-188 in bf16).
 */
int nf4b_dequantize(const nf4b_weight* w, void* out, void* stream);

/*
 * y = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * weight) over the last axis of
 * x[rows, width]. Replaces fusedops.rms_norm (app/engine/fusedops.py:61-95,
 * :169-196).
 */
int nf4b_rms_norm(const void* x, const void* weight, void* y, int rows, int width, float eps,
                  void* stream);

/*
 * Interleaved-pair rotary embedding of x[batch, seq, heads, head_dim] against
 * freqs[seq, head_dim/2, 2] = (cos, sin) of type freqs_dtype. Bit-exact to the
 * unfused fp32 formula. Replaces fusedops.rope (app/engine/fusedops.py:103-132,
 * :199-236).
 */
int nf4b_rope(const void* x, const void* freqs, int freqs_dtype, void* y, int batch, int seq,
              int heads, int head_dim, void* stream);

/*
 * One decode position: optional per-head RMSNorm of q and k (q_norm_w/k_norm_w
 * may be NULL), rotary on q and k, q -> q_out[n_head, head_dim], k and v into
 * the caches [n_kv, max_len, head_dim] at row *pos (read on the device, so a
 * captured graph serves every position). Replaces fusedlayer's `qk_rope_kv`
 * (app/engine/fusedlayer.py:56-92). head_dim must be 128.
 */
int nf4b_qk_rope_kv(const void* qkv, const void* q_norm_w, const void* k_norm_w, float eps,
                    const void* freqs, int freqs_dtype, const int64_t* pos, void* q_out,
                    void* k_cache, void* v_cache, int n_head, int n_kv, int head_dim, int max_len,
                    void* stream);

/*
 * Grouped-query attention of one query position over cache rows [0, L) with
 * L = min(*pos + 1, window) when `pos` is given (read on the device, so one
 * captured graph serves every position) and L = window otherwise; rows whose
 * `mask` byte is 0 are skipped (mask may be NULL = all visible). Query head h
 * reads KV head h / (n_head / n_kv). Caches are [n_kv, max_len, head_dim]
 * (max_len = the head stride in rows). out is bf16 [n_head, head_dim].
 * Replaces fusedlayer's attn_partial + attn_combine (app/engine/fusedlayer.py:95-157)
 * and fastpath.decode_attention for one query (app/engine/fastpath.py:133-174).
 * `workspace` must hold nf4b_decode_attention_workspace_size(...) bytes, zeroed
 * once before first use; calls leave it zeroed.
 */
int nf4b_decode_attention(const void* q, const void* k_cache, const void* v_cache,
                          const int64_t* pos, const uint8_t* mask, void* out, int n_head, int n_kv,
                          int head_dim, int max_len, int window, void* workspace,
                          size_t workspace_bytes, void* stream);

size_t nf4b_decode_attention_workspace_size(int n_head, int head_dim, int window);

/*
 * nf4b_qk_rope_kv then nf4b_decode_attention (pos given, no mask) in ONE
 * launch: the attention kernel reads q, k, v straight from the wqkv output,
 * applies the q/k norm and rotary with nf4b_qk_rope_kv's arithmetic, writes
 * the new k, v rows to the caches at *pos and attends over rows
 * [0, min(*pos + 1, window)) - the reference's qk_rope_kv + attn_partial +
 * attn_combine (app/engine/fusedlayer.py:56-157) as one call, results equal to
 * the two separate calls. Where the device cannot make the attention cluster
 * resident it issues the two calls, using q_scratch (n_head * head_dim bf16)
 * for the rotated q. Arguments as those two functions; workspace as
 * nf4b_decode_attention. No reference counterpart as a single call.
 */
int nf4b_qkv_attention(const void* qkv, const void* q_norm_w, const void* k_norm_w, float eps,
                       const void* freqs, int freqs_dtype, const int64_t* pos, void* q_scratch,
                       void* k_cache, void* v_cache, void* out, int n_head, int n_kv, int head_dim, int max_len,
                       int window, void* workspace, size_t workspace_bytes, void* stream);

/*
 * The elementwise calls above with the activation type as an argument: dtype
 * NF4B_BF16 (what the calls without _ex do) or NF4B_F16 - the reference's own
 * kernels are fp16 (app/engine/fusedops.py:61-132, app/engine/fusedlayer.py:
 * 56-157) - for x / y / weights / q / caches / out alike; the rotary table
 * keeps its own freqs_dtype. fp16 uses the same formulas with fp16 at every
 * rounding point. Any other dtype: NF4B_ERR_DTYPE.
 */
int nf4b_rms_norm_ex(const void* x, const void* weight, void* y, int rows, int width, float eps, int dtype,
                     void* stream);
int nf4b_rope_ex(const void* x, const void* freqs, int freqs_dtype, void* y, int batch, int seq,
                 int heads, int head_dim, int dtype, void* stream);
int nf4b_qk_rope_kv_ex(const void* qkv, const void* q_norm_w, const void* k_norm_w, float eps,
                       const void* freqs, int freqs_dtype, const int64_t* pos, void* q_out,
                       void* k_cache, void* v_cache, int n_head, int n_kv, int head_dim, int max_len,
                       int dtype, void* stream);
int nf4b_decode_attention_ex(const void* q, const void* k_cache, const void* v_cache,
                             const int64_t* pos, const uint8_t* mask, void* out, int n_head, int n_kv,
                             int head_dim, int max_len, int window, void* workspace,
                             size_t workspace_bytes, int dtype, void* stream);
int nf4b_qkv_attention_ex(const void* qkv, const void* q_norm_w, const void* k_norm_w, float eps,
                          const void* freqs, int freqs_dtype, const int64_t* pos, void* q_scratch,
                          void* k_cache, void* v_cache, void* out, int n_head, int n_kv, int head_dim,
                          int max_len, int window, void* workspace, size_t workspace_bytes, int dtype,
                          void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NF4B200_H */
