// Host-side declarations shared by the kernel files and the C ABI (capi.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "nf4b200.h"

namespace nf4b {

// ---- streaming GEMV (nf4_gemv.cu) ----------------------------------------

#ifndef NF4B_GEMV_WARPS
#define NF4B_GEMV_WARPS 8
#endif
#ifndef NF4B_GEMV_CTAS
#define NF4B_GEMV_CTAS 2
#endif
constexpr int GEMV_WARPS = NF4B_GEMV_WARPS;    // warps per CTA
constexpr int GEMV_CTAS_PER_SM = NF4B_GEMV_CTAS;  // persistent grid: CTAs per SM
constexpr int GEMV_LUT_BYTES = 256 * 256;      // pair table, 256 B stride, one copy per lane
constexpr int GEMV_SMEM_BYTES = GEMV_LUT_BYTES + 256 * 4;  // + code2 copy
// Pair kernel: one CTA of GEMV_PAIR_WARPS warps per SM. Shared memory: the pair
// table, code2 of W and of a gated pair's W3, each warp's ring of
// unit stages (a 16-row weight box written by TMA, 8 bytes of scale data per
// row and 128-code sub-unit written by cp.async, one mbarrier), then x staged
// whole when it fits (rows * k_in * 2 <= GEMV_PAIR_X_MAX).
#ifndef NF4B_GEMV_PAIR_WARPS
#define NF4B_GEMV_PAIR_WARPS 16
#endif
#ifndef NF4B_GEMV_PAIR_STAGE_KB
#define NF4B_GEMV_PAIR_STAGE_KB 6  // KB of weight ring per warp (stages = this / unit KB)
#endif
constexpr int GEMV_PAIR_WARPS = NF4B_GEMV_PAIR_WARPS;
constexpr int GEMV_PAIR_STAGE_KB = NF4B_GEMV_PAIR_STAGE_KB;
constexpr int GEMV_PAIR_SLOTS = GEMV_PAIR_WARPS * GEMV_PAIR_STAGE_KB;  // 1 KB weight slots
constexpr int GEMV_PAIR_W_OFFSET = GEMV_LUT_BYTES + 2 * 256 * 4;           // 1024-aligned boxes
constexpr int GEMV_PAIR_SC_OFFSET = GEMV_PAIR_W_OFFSET + GEMV_PAIR_SLOTS * 1024;
constexpr int GEMV_PAIR_BAR_OFFSET = GEMV_PAIR_SC_OFFSET + GEMV_PAIR_SLOTS * 128;
constexpr int GEMV_PAIR_X_OFFSET = GEMV_PAIR_BAR_OFFSET + GEMV_PAIR_SLOTS * 8;
#ifndef NF4B_GEMV_PAIR_X_KB
#define NF4B_GEMV_PAIR_X_KB 40
#endif
constexpr int GEMV_PAIR_X_MAX = NF4B_GEMV_PAIR_X_KB * 1024;
constexpr int GEMV_PAIR_SMEM_MAX = GEMV_PAIR_X_OFFSET + GEMV_PAIR_X_MAX;
static_assert(GEMV_PAIR_W_OFFSET % 1024 == 0, "TMA boxes must be aligned");
static_assert(GEMV_PAIR_SMEM_MAX <= 227 * 1024, "pair kernel shared memory exceeds one CTA's limit");
// Register-fed pair kernel: the pair table, then x of <= GEMV_REG_MAX_ROWS
// rows (rows * k_in * 2 <= GEMV_REG_X_MAX bytes, chunk-rotated, no padding).
// The GEMV chain's register-fed variant stages x with 16 bytes of padding per
// 128 and 64 per row (reg_x_row_bytes) under the same dynamic limit.
constexpr int GEMV_REG_SMEM_MAX = 227 * 1024 - 1024;  // 1 KB left for static shared memory
constexpr int GEMV_REG_X_MAX = GEMV_REG_SMEM_MAX - GEMV_LUT_BYTES;
constexpr int GEMV_REG_MAX_ROWS = 8;
static_assert(GEMV_LUT_BYTES + GEMV_PAIR_X_MAX * 9 / 8 + 128 <= GEMV_REG_SMEM_MAX, "chain staging exceeds the limit");
constexpr int GEMV_MAX_ROWS = 32;              // activation rows one launch takes
// The workspace starts with a fixed-size region of per-tile arrival counters,
// so calls on weights of different shapes never alias one another's counters
// with their partial sums. 16384 tiles of 16 rows: n_out <= 262144.
constexpr size_t GEMV_COUNTER_BYTES = 64 * 1024;
constexpr long long GEMV_MAX_TILES = GEMV_COUNTER_BYTES / 4;

// Byte ranges (16-byte aligned, whole 16-byte chunks) that a launch streams
// into L2 for later launches: packed codes and first-level scales of up to
// two weights. Each warp of the persistent grid takes an equal share.
struct PrefetchHint {
  const uint8_t* ptr[4];
  long long bytes[4];
};

// Warp gw's share (of W) of every hinted range, streamed into L2 with bulk
// prefetches (fire and forget; at most 32 KB each).
__device__ __forceinline__ void prefetch_share(const PrefetchHint& h, long long gw, long long W) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const long long chunks = h.bytes[i] >> 4;
    if (chunks <= 0) continue;
    const long long a = (gw * chunks / W) << 4, b = ((gw + 1) * chunks / W) << 4;
    const char* ptr = reinterpret_cast<const char*>(h.ptr[i]) + a;
    for (long long left = b - a; left > 0;) {
      const uint32_t n = left > 32768 ? 32768u : (uint32_t)left;
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(ptr), "r"(n) : "memory");
      ptr += n;
      left -= n;
    }
  }
}

struct alignas(64) GemvParams {
  const uint8_t* packed;
  const uint8_t* a8;
  const float* absmax;
  const float* code2;
  float offset;
  // Gated pair (pair kernel only): W3, same shape and quantisation as W; the
  // output is the FeedForward gate of x W^T and x W3^T. code2_3 is null otherwise.
  const uint8_t* packed3;
  const uint8_t* a8_3;
  const float* absmax3;
  const float* code2_3;
  float offset3;
  int gated;
  int su;        // pair kernel: 128-code sub-units per unit (1 or 2)
  int reg;       // su == 2, rows <= 2: the register-fed pair kernel (weights loaded straight into registers)
  int f16;       // fp16 x, operand, y and norm weight (register-fed kernel only); else bf16
  int x_staged;  // pair kernel: x is copied whole into shared memory first
  const uint16_t* norm_w;  // pair kernel, staged x: RMS-normalise x with this weight first (or null)
  float norm_eps;
  // Pair kernel: TMA maps of the packed weights (W, and W3 of a gated pair) as
  // [n_out rows, k_in / 2 bytes], boxes of 64 bytes x 16 rows.
  CUtensorMap wmap;
  CUtensorMap wmap3;
  int N, K;
  int nested;
  int bs_shift;
  int bs2_shift;
  const uint16_t* x;
  uint16_t* y;
  const uint16_t* operand;
  int M;
  int epi;
  float* partial;
  int* counters;
  long long units;
  int warps_total;
  int blocks_per_tile;
  // Warp w owns units [w*uq + min(w, ur), (w+1)*uq + min(w+1, ur)): uq = units /
  // warps, ur = units % warps (computed on the host; 32-bit arithmetic on the device).
  int uq, ur;
  // Optional L2 prefetch of the weight the NEXT call reads (packed codes and
  // its first-level scales), issued by each warp once its own loads are done.
  PrefetchHint pf;
  // Rotary + KV-cache write fused into the store (register-fed kernel, one
  // activation row, no q/k norm; rk_q null otherwise). Output rows are rk_nh
  // query heads, then rk_nkv key heads, then rk_nkv value heads of 128.
  const void* rk_freqs;  // this token's rotary row: 128 values, (cos, sin) pairs
  int rk_ftype;
  const int64_t* rk_pos;
  uint16_t* rk_q;
  uint16_t* rk_k;
  uint16_t* rk_v;
  int rk_nh, rk_nkv, rk_max_len;
};

struct GemvPlan {
  long long tiles;
  long long units;
  int blocks_per_tile;  // units per row tile (k_in / 128 for the pair kernel, / 64 otherwise)
  int warps_total;
  int grid;
  int slots;
  size_t counter_bytes;
  size_t partial_bytes;
};

int gemv_sm_count(int dev);
// `pairs`: use the pair kernel (units of 128 codes; up to 4 activation rows,
// k_in % 128 == 0, scale arrays aligned for its paired loads).
// `gated`: the pair kernel's gated mode (tiles of W units then W3 units).
// `su`: 128-code sub-units per pair-kernel unit (2 for blocksize-64 weights
// with k_in % 256 == 0 whose x fits the shared-memory stage, else 1).
void gemv_plan(int N, int K, int M, int sm_count, bool pairs, GemvPlan* plan, bool gated = false, int su = 1);
cudaError_t launch_gemv(const GemvParams& p, int grid, bool pairs, cudaStream_t stream);

// ---- GEMV chain (nf4_gemv.cu): dependent decode GEMVs in one persistent launch

constexpr int CHAIN_MAX_JOBS = 40;
// The done counters (one per job) and the CTA exit counter sit at the end of
// the workspace's counter region; split-tile counters use its start.
constexpr int CHAIN_DONE_INTS = 64;
constexpr long long CHAIN_MAX_TILES = GEMV_MAX_TILES - CHAIN_DONE_INTS;

struct alignas(64) ChainJob {
  CUtensorMap wmap;   // packed W, boxes of 128 bytes x 16 rows
  CUtensorMap wmap3;  // gated pair: W3
  const uint8_t* packed;   // the register-fed chain reads the packed weights directly
  const uint8_t* packed3;
  const uint8_t* a8;
  const float* absmax;
  const float* code2;
  const uint8_t* a8_3;
  const float* absmax3;
  const float* code2_3;
  const uint16_t* x;
  uint16_t* y;
  const uint16_t* operand;
  const uint16_t* norm_w;  // RMS-normalise x with this weight first, or null
  float offset, offset3, norm_eps;
  int N, K;
  int nested, bs2_shift, gated, epi;
  int B;      // 256-code units per row tile and half
  int tiles;  // row tiles of 16
  int uq, ur; // warp w's run: [w*uq + min(w, ur), ...) of tiles * B * (gated ? 2 : 1) units
};

struct alignas(64) ChainParams {
  int n_jobs;
  int M;
  int reg;  // rows <= 2 and every job's weights 32-byte aligned: the register-fed chain
  int warps_total;
  float* partial;
  int* counters;
  ChainJob jobs[CHAIN_MAX_JOBS];
};

// Units and warp runs of every job (fields B, tiles, uq, ur); returns the
// partial-sum bytes the split tiles need (the largest job's).
size_t chain_plan(ChainParams* p, int sm_count);
cudaError_t launch_gemv_chain(const ChainParams& p, cudaStream_t stream);

// ---- persistent decode step (decode_step.cu): dependent decode GEMVs in one
// cooperative launch, handing outputs over through flag-tagged 64-bit words

constexpr int STEP_WARPS = 16;
constexpr int STEP_MAX_JOBS = NF4B_MAX_STEP_JOBS;
constexpr int STEP_MAX_K = 10240;            // x of 2 rows staged whole in shared memory
constexpr size_t STEP_CONTROL_BYTES = 256;   // epoch (u32) and exit counter (i32), padded

struct StepJob {
  const uint8_t* packed;
  const uint8_t* a8;
  const float* absmax;
  const float* code2;
  const uint8_t* packed3;  // gated pair: W3 (same shape and quantisation)
  const uint8_t* a8_3;
  const float* absmax3;
  const float* code2_3;
  const uint16_t* x;
  uint16_t* y;
  const uint16_t* operand;
  const uint16_t* norm_w;
  float offset, offset3, norm_eps;
  int N, K;
  int nested, gated, epi, bs2_shift;
  // derived by step_plan
  int B;        // 256-code units per row tile and half
  int tiles;    // row tiles of 16
  int units;    // tiles * B * (gated ? 2 : 1)
  int smax;     // the most CTAs one tile meets
  int x_ll;     // x is the previous job's y: staged from its handoff words
  int op_ll;    // 1 / 2: the epilogue operand is job j - op_ll's y, read from its handoff words (0: memory)
  int barrier;  // the boundary after this job is a full barrier (arrival words)
};

struct alignas(16) StepParams {
  int n_jobs;
  int M;
  int grid;
  int stall_job;                  // test hook: the boundary before this job never completes (-1: none)
  unsigned long long wait_ns;     // how long a wait lasts before it gives up
  long long ll_words;             // 64-bit handoff words per region
  uint64_t* ll[3];                // handoff regions, job j's in region j % 3
  uint64_t* arrive;               // [2][grid] arrival words
  unsigned* epoch;
  int* exit_ctr;
  StepJob jobs[STEP_MAX_JOBS];
};

// Fills the derived job fields and returns the workspace bytes the step needs.
size_t step_plan(StepParams* p, int sm_count);
cudaError_t launch_decode_step(StepParams& p, void* workspace, cudaStream_t stream);
int read_step_error(int clear);

// ---- dense bf16 GEMV for the output heads (dense_gemv.cu) -----------------
// k_in in {1024, 2048, 2560, 4096}; one activation row.
cudaError_t launch_dense_gemv(const uint16_t* w, const uint16_t* x, uint16_t* y, int n_out, int k_in, int sms,
                              const uint16_t* norm_w, float norm_eps, cudaStream_t stream);

// ---- Dual-AR frame bookkeeping (frame_ops.cu) -------------------------------
constexpr int FRAME_MAX_CODEBOOKS = 32;
cudaError_t launch_embed_rows(const uint16_t* table, long long rows, const int64_t* ids, int n_ids, int dim,
                              uint16_t* out, cudaStream_t stream);
cudaError_t launch_frame_select(const int64_t* main_tok, const int64_t* high_tok, const int64_t* recent,
                                int n_recent, long long sem_begin, long long cb_size, int64_t* tokens,
                                const uint16_t* fast_emb, int dim, uint16_t* h, cudaStream_t stream);
cudaError_t launch_frame_advance(const uint16_t* sem_emb, long long vocab, const uint16_t* cb_emb, long long cb_size,
                                 int n_cb, const int64_t* tokens, int dim, uint16_t* x, int64_t* recent,
                                 int n_recent, int64_t* pos, int64_t* step, cudaStream_t stream);

// ---- fused top-k / top-p sampler (sampler.cu) -------------------------------
// V <= 8192 * 2048 / 64 logits (the last CTA sorts <= 8192 slice winners).
constexpr int SAMPLER_MAX_VOCAB = 262144;
size_t sampler_workspace_bytes(int V);
cudaError_t launch_sampler(const uint16_t* logits, int V, float temperature, float top_p, int top_k,
                           unsigned long long seed, const int64_t* step, int64_t* out, void* workspace,
                           cudaStream_t stream);

// ---- dequantisation (nf4_dequant.cu) ---------------------------------------

struct DequantParams {
  const uint8_t* packed;
  const uint8_t* a8;
  const float* absmax;
  const float* code2;
  float offset;
  int N, K;
  int nested;
  int bs_shift;
  int bs2_shift;
  uint16_t* out;
};
cudaError_t launch_dequant(const DequantParams& p, cudaStream_t stream);

// ---- tcgen05 GEMM (nf4_gemm_tc.cu) -----------------------------------------

struct GemmParams {
  const uint8_t* packed;
  const uint8_t* a8;
  const float* absmax;
  const float* code2;
  float offset;
  int N, K;
  int nested;
  int bs_shift;
  int bs2_shift;
  const uint16_t* x;
  uint16_t* y;
  const uint16_t* operand;
  int M;
  int epi;
  // split-K (grid z = splits > 1): fp32 partial sums [splits, M, N] and one
  // counter per output tile; the last CTA of a tile sums the splits in order
  int splits;
  float* partial;
  int* counters;
  int bt;  // activation rows per tile: gemm_bt(N, M, K, sms)
  int f16;  // fp16 x, operand and y; else bf16
};
constexpr size_t GEMM_COUNTER_BYTES = 4096;  // tile counters of a split-K launch (<= 1024 tiles)
// Split-K factor the GEMM would use for this shape on `sms` SMs (1: none), and
// the workspace it then needs (0 when 1).
int gemm_bt(int N, int M, int K, int sms);
int gemm_splits(int N, int M, int K, int sms);
size_t gemm_workspace_bytes(int N, int M, int K, int sms);
cudaError_t launch_gemm_tc(const GemmParams& p, cudaStream_t stream);

// ---- fused elementwise (fused_ops.cu) -------------------------------------
// f16: fp16 activations and weights (the reference's dtype); else bf16.

cudaError_t launch_rms_norm(const uint16_t* x, const uint16_t* w, uint16_t* y, int rows,
                            int width, float eps, cudaStream_t stream, bool f16 = false);
cudaError_t launch_rope(const uint16_t* x, const void* freqs, int ftype, uint16_t* y,
                        long long pairs, int half_dim, int heads, int seq, cudaStream_t stream,
                        bool f16 = false);
cudaError_t launch_qk_rope_kv(const uint16_t* qkv, const uint16_t* qw, const uint16_t* kw,
                              float eps, const void* freqs, int ftype, const int64_t* pos,
                              uint16_t* q_out, uint16_t* kc, uint16_t* vc, int nh, int nkv,
                              int max_len, cudaStream_t stream, bool f16 = false);

// ---- decode attention (decode_attention.cu) ---------------------------------

constexpr int ATTN_CHUNK = 64;  // cache rows per CTA
constexpr size_t ATTN_COUNTER_BYTES = 4096;  // fixed counter region: up to 1024 KV heads
struct AttnPlan {
  int chunks;
  size_t counter_bytes;
  size_t partial_bytes;
};
void attn_plan(int n_head, int head_dim, int window, AttnPlan* plan);
// One thread-block cluster of 8 CTAs per KV head; cudaErrorNotSupported when
// such a cluster cannot be resident on the device.
struct QkvIn;
cudaError_t launch_cluster_attention(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int64_t* pos,
                                     const uint8_t* mask, uint16_t* out, int nh, int nkv, int max_len, int window,
                                     cudaStream_t stream, const QkvIn& in, bool f16 = false);
cudaError_t launch_decode_attention(const uint16_t* q, const uint16_t* kc, const uint16_t* vc,
                                    const int64_t* pos, const uint8_t* mask, uint16_t* out, int nh, int nkv,
                                    int max_len, int window, float* partial, int* counters,
                                    cudaStream_t stream, bool f16 = false);
// The decode step's q/k norm + rotary + KV write (qk_rope_kv's arithmetic)
// taken by the cluster attention kernel from the wqkv output directly.
struct QkvIn {
  const uint16_t* qkv;  // [n_head + 2 n_kv, 128] bf16
  const uint16_t* qw;   // q_norm weight [128] or null
  const uint16_t* kw;   // k_norm weight [128] or null
  float eps;
  const void* freqs;    // the position's rotary row [64, 2]
  int ftype;
  int n_head;
};
// One launch when a cluster can be resident; otherwise launch_qk_rope_kv into
// q_scratch then launch_decode_attention (needs partial/counters).
cudaError_t launch_qkv_attention(const QkvIn& in, const int64_t* pos, uint16_t* q_scratch, uint16_t* kc,
                                 uint16_t* vc, uint16_t* out, int nh, int nkv, int max_len, int window,
                                 float* partial, int* counters, cudaStream_t stream, bool f16 = false);

}  // namespace nf4b
