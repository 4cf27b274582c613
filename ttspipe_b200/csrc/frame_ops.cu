// Dual-AR frame bookkeeping on the device (sm_100a): the token logic between a
// frame's samplers and its next input, which would otherwise be a dozen tiny
// framework launches per frame (compares, reductions, gathers, copies).
//
// The frame (ttspipe_b200.dualar) follows the reference's captured decode step
// (app/engine/graphs.py:105-127): the semantic token is replaced by the
// high-temperature draw when it is a semantic id that occurs in the recent
// window (repetition-aware sampling), the fast AR is fed the embedding of
// each drawn code, and the next frame's input is the semantic embedding plus
// the codebook embeddings of the frame's codes (app/engine/hostembed.py:3-4).

#include "common.cuh"
#include "kernels.cuh"

namespace nf4b {

namespace {

constexpr int kFrameThreads = 256;

__device__ __forceinline__ long long clamp_ll(long long v, long long lo, long long hi) {
  return v < lo ? lo : (v > hi ? hi : v);
}

// dst[0..dim) = src[0..dim) in 16-byte pieces (dim % 8 == 0, both 16-byte aligned).
__device__ __forceinline__ void copy_row(const uint16_t* src, uint16_t* dst, int dim) {
  for (int i = threadIdx.x; i < dim / 8; i += kFrameThreads)
    reinterpret_cast<uint4*>(dst)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
}

// out row r = table row ids[r] (clamped to the table).
__global__ void __launch_bounds__(kFrameThreads)
    embed_rows_kernel(const uint16_t* __restrict__ table, long long rows, const int64_t* __restrict__ ids, int dim,
                      uint16_t* __restrict__ out) {
  pdl_wait();  // the ids come from the previous kernel (a sampler)
  const long long id = clamp_ll(ids[blockIdx.x], 0, rows - 1);
  copy_row(table + id * dim, out + (size_t)blockIdx.x * dim, dim);
  pdl_launch_dependents();
}

// main' = high if main is a semantic id (sem_begin <= main < sem_begin +
// cb_size) that occurs in recent[0..n_recent), else main; tokens[0] = main';
// tokens[1] = a = clamp(main' - sem_begin, 0, cb_size - 1); h = fast_emb row a.
__global__ void __launch_bounds__(kFrameThreads)
    frame_select_kernel(const int64_t* __restrict__ main_tok, const int64_t* __restrict__ high_tok,
                        const int64_t* __restrict__ recent, int n_recent, long long sem_begin, long long cb_size,
                        int64_t* __restrict__ tokens, const uint16_t* __restrict__ fast_emb, int dim,
                        uint16_t* __restrict__ h) {
  __shared__ long long s_a;
  pdl_wait();
  if (threadIdx.x == 0) {
    const long long m = main_tok[0];
    bool seen = false;
    for (int j = 0; j < n_recent; ++j) seen |= recent[j] == m;
    const bool semantic = m >= sem_begin && m < sem_begin + cb_size;
    const long long chosen = (seen && semantic) ? high_tok[0] : m;
    const long long a = clamp_ll(chosen - sem_begin, 0, cb_size - 1);
    tokens[0] = chosen;
    tokens[1] = a;
    s_a = a;
  }
  __syncthreads();
  copy_row(fast_emb + s_a * dim, h, dim);
  pdl_launch_dependents();
}

// x = bf16(float(sem_emb[tokens[0]]) + s), s = the fp32 sum, in codebook
// order, of float(cb_emb[i][tokens[1 + i]]) for i < n_cb; recent <-
// [tokens[0], recent[0..n_recent-2]]; pos += 1; step += 1. One thread per
// dimension (CTA b takes dimensions b * 256 ..); CTA 0 moves the counters.
__global__ void __launch_bounds__(kFrameThreads)
    frame_advance_kernel(const uint16_t* __restrict__ sem_emb, long long vocab, const uint16_t* __restrict__ cb_emb,
                         long long cb_size, int n_cb, const int64_t* __restrict__ tokens, int dim,
                         uint16_t* __restrict__ x, int64_t* __restrict__ recent, int n_recent,
                         int64_t* __restrict__ pos, int64_t* __restrict__ step) {
  __shared__ long long s_tok[FRAME_MAX_CODEBOOKS + 1];
  pdl_wait();
  if (threadIdx.x <= n_cb)
    s_tok[threadIdx.x] = clamp_ll(tokens[threadIdx.x], 0, (threadIdx.x == 0 ? vocab : cb_size) - 1);
  __syncthreads();
  const int d = blockIdx.x * kFrameThreads + threadIdx.x;
  if (d < dim) {
    // every row's element requested before the sum (one round trip)
    float e[FRAME_MAX_CODEBOOKS];
#pragma unroll
    for (int i = 0; i < FRAME_MAX_CODEBOOKS; ++i)
      e[i] = i < n_cb ? bf2f(cb_emb[((size_t)i * cb_size + s_tok[1 + i]) * dim + d]) : 0.f;
    const float sem = bf2f(sem_emb[(size_t)s_tok[0] * dim + d]);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < FRAME_MAX_CODEBOOKS; ++i)
      if (i < n_cb) s += e[i];
    x[d] = f2bf(__fadd_rn(sem, s));
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    for (int j = n_recent - 1; j > 0; --j) recent[j] = recent[j - 1];
    if (n_recent > 0) recent[0] = s_tok[0];
    pos[0] += 1;
    step[0] += 1;
  }
  pdl_launch_dependents();
}

cudaError_t launch_frame_kernel(const void* fn, int grid, void** args, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kFrameThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace

cudaError_t launch_embed_rows(const uint16_t* table, long long rows, const int64_t* ids, int n_ids, int dim,
                              uint16_t* out, cudaStream_t stream) {
  void* args[] = {(void*)&table, (void*)&rows, (void*)&ids, (void*)&dim, (void*)&out};
  return launch_frame_kernel((const void*)embed_rows_kernel, n_ids, args, stream);
}

cudaError_t launch_frame_select(const int64_t* main_tok, const int64_t* high_tok, const int64_t* recent,
                                int n_recent, long long sem_begin, long long cb_size, int64_t* tokens,
                                const uint16_t* fast_emb, int dim, uint16_t* h, cudaStream_t stream) {
  void* args[] = {(void*)&main_tok, (void*)&high_tok, (void*)&recent,   (void*)&n_recent, (void*)&sem_begin,
                  (void*)&cb_size,  (void*)&tokens,   (void*)&fast_emb, (void*)&dim,      (void*)&h};
  return launch_frame_kernel((const void*)frame_select_kernel, 1, args, stream);
}

cudaError_t launch_frame_advance(const uint16_t* sem_emb, long long vocab, const uint16_t* cb_emb, long long cb_size,
                                 int n_cb, const int64_t* tokens, int dim, uint16_t* x, int64_t* recent,
                                 int n_recent, int64_t* pos, int64_t* step, cudaStream_t stream) {
  void* args[] = {(void*)&sem_emb, (void*)&vocab, (void*)&cb_emb, (void*)&cb_size,  (void*)&n_cb, (void*)&tokens,
                  (void*)&dim,     (void*)&x,     (void*)&recent, (void*)&n_recent, (void*)&pos,  (void*)&step};
  return launch_frame_kernel((const void*)frame_advance_kernel, (dim + kFrameThreads - 1) / kFrameThreads, args,
                             stream);
}

}  // namespace nf4b
