// Grouped-query decode attention for one query position over a bf16 KV cache.
//
// Replaces the reference's split-K pair attn_partial + attn_combine
// (app/engine/fusedlayer.py:95-157) with one launch. Grid (n_kv, chunks): each
// CTA reads ATTN_CHUNK cache rows of one KV head ONCE for all query heads of
// its group (query head h reads KV head h / groups, the grouping of
// app/engine/fastpath.py:156-170), and keeps an fp32 online-softmax partial
// (max, sum, unnormalised output). The last CTA of a KV head to finish (atomic
// counter, reset after use) merges the partials in chunk order and writes the
// bf16 output - no second launch, no spin-wait. The live length comes from the
// device-side position (*pos + 1), so one captured graph serves every position
// up to `window`; chunks past the live length exit at once.
//
// Scores follow the fork's rounding: bf16(q.k) * head_dim^-0.5 in fp32.

#include "common.cuh"
#include "kernels.cuh"

namespace nf4b {

namespace {

constexpr int kD = 128;
constexpr int kThreads = 128;

template <int G>
__global__ void __launch_bounds__(kThreads) decode_attention_kernel(
    const bf16_t* __restrict__ q, const bf16_t* __restrict__ kc, const bf16_t* __restrict__ vc,
    const int64_t* __restrict__ pos_ptr, const uint8_t* __restrict__ mask, bf16_t* __restrict__ out,
    int max_len, int window,
    int chunks, float scale, float* __restrict__ part_acc, float* __restrict__ part_ml,
    int* __restrict__ counters) {
  __shared__ float q_s[G][kD];
  __shared__ float sc_s[G][ATTN_CHUNK];
  __shared__ float m_s[G], l_s[G];
  __shared__ float red[4][G][kD];
  __shared__ int last_s;

  pdl_wait();
  const int kh = blockIdx.x, c = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  long long L = (pos_ptr != nullptr) ? pos_ptr[0] + 1 : (long long)window;
  if (L > window) L = window;
  if (L < 1) L = 1;
  const int active = (int)((L + ATTN_CHUNK - 1) / ATTN_CHUNK);
  if (c >= active) {
    pdl_launch_dependents();
    return;
  }
  const long long j0 = (long long)c * ATTN_CHUNK;
  const bf16_t* kbase = kc + (size_t)kh * max_len * kD;
  const bf16_t* vbase = vc + (size_t)kh * max_len * kD;

  for (int i = tid; i < G * kD; i += kThreads) q_s[i / kD][i % kD] = bf2f(q[(size_t)kh * G * kD + i]);
  __syncthreads();

  // Scores: a warp takes 16 rows, four at a time, eight lanes per row and
  // sixteen dimensions per lane.
  {
    const int gi = lane >> 3, li = lane & 7;
    for (int it = 0; it < 4; ++it) {
      const int jl = warp * 16 + it * 4 + gi;
      const long long j = j0 + jl;
      float dot[G];
#pragma unroll
      for (int h = 0; h < G; ++h) dot[h] = 0.f;
      const bool vis = (j < L) && (mask == nullptr || mask[j] != 0);
      if (vis) {
        const uint4* kr = reinterpret_cast<const uint4*>(kbase + (size_t)j * kD + li * 16);
        const uint4 k0 = __ldg(kr), k1 = __ldg(kr + 1);
        const uint32_t kw[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float ka = __uint_as_float(kw[e] << 16), kb = __uint_as_float(kw[e] & 0xFFFF0000u);
#pragma unroll
          for (int h = 0; h < G; ++h) {
            dot[h] = fmaf(q_s[h][li * 16 + 2 * e], ka, dot[h]);
            dot[h] = fmaf(q_s[h][li * 16 + 2 * e + 1], kb, dot[h]);
          }
        }
      }
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float v = dot[h];
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        if (li == 0) sc_s[h][jl] = vis ? __fmul_rn(round_bf(v), scale) : -INFINITY;
      }
    }
  }
  __syncthreads();

  // Chunk max and exp per head (a warp per head).
  for (int h = warp; h < G; h += 4) {
    const float a = sc_s[h][lane], b = sc_s[h][lane + 32];
    float m = fmaxf(a, b);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    const float pa = (a == -INFINITY) ? 0.f : expf(a - m);
    const float pb = (b == -INFINITY) ? 0.f : expf(b - m);
    sc_s[h][lane] = pa;
    sc_s[h][lane + 32] = pb;
    float l = pa + pb;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    if (lane == 0) {
      m_s[h] = m;
      l_s[h] = l;
    }
  }
  __syncthreads();

  // P.V: 16 dimension groups of 8 x 8 row groups of 8.
  {
    const int dg = tid & 15, pg = tid >> 4;
    float acc[G][8];
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[h][e] = 0.f;
    for (int r = 0; r < 8; ++r) {
      const int jl = pg * 8 + r;
      const long long j = j0 + jl;
      if (j >= L) break;
      if (mask != nullptr && mask[j] == 0) continue;  // masked rows are never read
      const uint4 vv = __ldg(reinterpret_cast<const uint4*>(vbase + (size_t)j * kD + dg * 8));
      const uint32_t vw[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float p = sc_s[h][jl];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          acc[h][2 * e] = fmaf(p, __uint_as_float(vw[e] << 16), acc[h][2 * e]);
          acc[h][2 * e + 1] = fmaf(p, __uint_as_float(vw[e] & 0xFFFF0000u), acc[h][2 * e + 1]);
        }
      }
    }
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float v = acc[h][e] + __shfl_xor_sync(0xffffffffu, acc[h][e], 16);
        if ((lane & 16) == 0) red[warp][h][dg * 8 + e] = v;
      }
  }
  __syncthreads();
  for (int i = tid; i < G * kD; i += kThreads) {
    const int h = i / kD, d = i % kD;
    const float v = red[0][h][d] + red[1][h][d] + red[2][h][d] + red[3][h][d];
    const int qh = kh * G + h;
    part_acc[((size_t)qh * chunks + c) * kD + d] = v;
  }
  if (tid < G) {
    const int qh = kh * G + tid;
    part_ml[((size_t)qh * chunks + c) * 2] = m_s[tid];
    part_ml[((size_t)qh * chunks + c) * 2 + 1] = l_s[tid];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int old = atomicAdd(counters + kh, 1);
    last_s = (old == active - 1);
    if (last_s) counters[kh] = 0;
  }
  __syncthreads();
  if (!last_s) {
    pdl_launch_dependents();
    return;
  }
  __threadfence();

  // Merge the chunk partials of every head of this group, in chunk order.
  for (int i = tid; i < G * kD; i += kThreads) {
    const int h = i / kD, d = i % kD;
    const int qh = kh * G + h;
    const float* ml = part_ml + (size_t)qh * chunks * 2;
    float M = -INFINITY;
    for (int cc = 0; cc < active; ++cc) M = fmaxf(M, __ldcg(ml + 2 * cc));
    float num = 0.f, den = 0.f;
    for (int cc = 0; cc < active; ++cc) {
      const float w = expf(__ldcg(ml + 2 * cc) - M);
      den = fmaf(__ldcg(ml + 2 * cc + 1), w, den);
      num = fmaf(__ldcg(part_acc + ((size_t)qh * chunks + cc) * kD + d), w, num);
    }
    out[(size_t)qh * kD + d] = f2bf(num / den);
  }
  pdl_launch_dependents();
}

}  // namespace

void attn_plan(int n_head, int head_dim, int window, AttnPlan* plan) {
  plan->chunks = (window + ATTN_CHUNK - 1) / ATTN_CHUNK;
  plan->counter_bytes = ATTN_COUNTER_BYTES;
  plan->partial_bytes = (size_t)n_head * plan->chunks * (head_dim + 2) * sizeof(float);
}

cudaError_t launch_decode_attention(const uint16_t* q, const uint16_t* kc, const uint16_t* vc,
                                    const int64_t* pos, const uint8_t* mask, uint16_t* out, int nh, int nkv,
                                    int max_len, int window, float* partial, int* counters,
                                    cudaStream_t stream) {
  const int groups = nh / nkv;
  const int chunks = (window + ATTN_CHUNK - 1) / ATTN_CHUNK;
  float* part_acc = partial;
  float* part_ml = partial + (size_t)nh * chunks * kD;
  const float scale = 1.0f / sqrtf((float)kD);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nkv, chunks);
  cfg.blockDim = dim3(kThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
#define NF4B_ATTN_CASE(GG)                                                                      \
  case GG:                                                                                      \
    return cudaLaunchKernelEx(&cfg, decode_attention_kernel<GG>, (const bf16_t*)q,             \
                              (const bf16_t*)kc, (const bf16_t*)vc, pos, mask, (bf16_t*)out, max_len, \
                              window, chunks, scale, part_acc, part_ml, counters);
  switch (groups) {
    NF4B_ATTN_CASE(1)
    NF4B_ATTN_CASE(2)
    NF4B_ATTN_CASE(4)
    NF4B_ATTN_CASE(8)
    default:
      return cudaErrorInvalidValue;
  }
#undef NF4B_ATTN_CASE
}

}  // namespace nf4b
