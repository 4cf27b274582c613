// Fused top-k / top-p sampling of one token from a bf16 logit row, on the
// device, graph-capturable: the semantics of the fork's sampler as the
// reference calls it (app/engine/graphs.py:55-73, fused in
// app/engine/fusedsample.py:44-257, top-k capped at 64 there too):
//
//   sort logits descending; p = softmax(sorted) over the WHOLE vocabulary;
//   drop position i when cumsum(p)[i] > top_p or i >= top_k (never i = 0);
//   divide the kept logits by max(temperature, 1e-5), softmax over them,
//   draw one.
//
// One launch. CTA s takes a 2048-logit slice (a vocabulary of up to 4096, the
// codebooks', is one CTA's, two slices, drawn at once): each of its 32 warps sorts 64
// (value, index) keys (larger value first, then smaller index) in registers,
// and the warps' lists are merged pairwise - the top 64 of two sorted lists
// is max(A[i], B[63 - i]), a bitonic sequence, then a 6-stage bitonic merge -
// down to the slice's 64 best, published with the slice's (max, sum of exp)
// for the full-vocabulary softmax. The last CTA (atomic counter, reset after
// use) merges the slices' lists the same way and draws. The draw is
// inverse-CDF with one uniform from a counter-based hash of (seed, *step) -
// the same distribution as the fork's exponential race, reproducible from the
// seed.

#include "common.cuh"
#include "kernels.cuh"

namespace nf4b {

namespace {

constexpr int kSlice = 2048;
constexpr int kSThreads = 1024;
constexpr int kTop = 64;
constexpr int kMaxSlices = (SAMPLER_MAX_VOCAB + kSlice - 1) / kSlice;
static_assert(kSThreads == 32 * 32 && kSlice == 64 * 32, "one 64-key list per warp, 32 warps");

__device__ __forceinline__ unsigned long long make_key(float v, uint32_t idx) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);  // order-preserving
  return ((unsigned long long)b << 32) | (0xFFFFFFFFu - idx);
}
__device__ __forceinline__ float key_value(unsigned long long k) {
  uint32_t b = (uint32_t)(k >> 32);
  b = (b & 0x80000000u) ? (b & 0x7FFFFFFFu) : ~b;
  return __uint_as_float(b);
}
__device__ __forceinline__ uint32_t key_index(unsigned long long k) { return 0xFFFFFFFFu - (uint32_t)k; }
// The same order in 32 bits for a one-CTA vocabulary (indices below 65536): the
// logit's bf16 bits (a bf16 value's low 16 fp32 bits are zero), then the index.
// Half the shuffles of the 64-bit key in the sorts and merges, which bound them.
__device__ __forceinline__ uint32_t make_key32(float v, uint32_t idx) {
  uint32_t b = __float_as_uint(v) >> 16;
  b = (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
  return (b << 16) | (0xFFFFu - idx);
}
__device__ __forceinline__ float key_value(uint32_t k) {
  uint32_t b = k >> 16;
  b = (b & 0x8000u) ? (b & 0x7FFFu) : (~b & 0xFFFFu);
  return __uint_as_float(b << 16);
}
__device__ __forceinline__ uint32_t key_index(uint32_t k) { return 0xFFFFu - (k & 0xFFFFu); }
template <typename Key>
__device__ __forceinline__ Key make_key_t(float v, uint32_t idx) {
  if constexpr (sizeof(Key) == 4)
    return make_key32(v, idx);
  else
    return make_key(v, idx);
}

// A sorted (descending) list of 64 keys held by one warp: lane l holds
// L[l] in x0 and L[l + 32] in x1.
template <typename Key>
__device__ __forceinline__ Key kmax(Key a, Key b) { return a > b ? a : b; }
template <typename Key>
__device__ __forceinline__ Key kmin(Key a, Key b) { return a < b ? a : b; }

// Sort 64 arbitrary keys into that layout (bitonic network; strides below 32
// between lanes, stride 32 within a lane).
template <typename Key>
__device__ __forceinline__ void warp_sort64(Key& x0, Key& x1, int lane) {
#pragma unroll
  for (int k = 2; k <= 64; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j == 32) {  // k == 64: element i against i + 32, descending
        const Key hi = kmax(x0, x1), lo = kmin(x0, x1);
        x0 = hi;
        x1 = lo;
        continue;
      }
      const bool lower = (lane & j) == 0;
      const bool d0 = (lane & k) == 0, d1 = ((lane + 32) & k) == 0;  // block of element i sorted descending?
      const Key p0 = __shfl_xor_sync(0xffffffffu, x0, j);
      const Key p1 = __shfl_xor_sync(0xffffffffu, x1, j);
      x0 = (lower == d0) ? kmax(x0, p0) : kmin(x0, p0);
      x1 = (lower == d1) ? kmax(x1, p1) : kmin(x1, p1);
    }
  }
}

// (a0, a1) <- the top 64 of the sorted lists A = (a0, a1) and B = (b0, b1), sorted.
template <typename Key>
__device__ __forceinline__ void warp_merge64(Key& a0, Key& a1, Key b0, Key b1, int lane) {
  const Key r0 = __shfl_sync(0xffffffffu, b1, 31 - lane);  // B[63 - lane]
  const Key r1 = __shfl_sync(0xffffffffu, b0, 31 - lane);  // B[31 - lane]
  Key c0 = kmax(a0, r0), c1 = kmax(a1, r1);              // bitonic
  const Key hi = kmax(c0, c1), lo = kmin(c0, c1);
  c0 = hi;
  c1 = lo;
#pragma unroll
  for (int j = 16; j > 0; j >>= 1) {
    const bool lower = (lane & j) == 0;
    const Key p0 = __shfl_xor_sync(0xffffffffu, c0, j);
    const Key p1 = __shfl_xor_sync(0xffffffffu, c1, j);
    c0 = lower ? kmax(c0, p0) : kmin(c0, p0);
    c1 = lower ? kmax(c1, p1) : kmin(c1, p1);
  }
  a0 = c0;
  a1 = c1;
}

// Merge the 32 warps' lists (registers) down to warp 0's; lists[32][64] is
// shared scratch. Leaves the result in lists[0] too. Every thread calls it.
template <typename Key>
__device__ __forceinline__ void block_merge(Key (*lists)[kTop], Key& x0, Key& x1, int warp, int lane) {
  lists[warp][lane] = x0;
  lists[warp][lane + 32] = x1;
#pragma unroll
  for (int lvl = 1; lvl < 32; lvl <<= 1) {
    __syncthreads();
    if ((warp & (2 * lvl - 1)) == 0) {
      warp_merge64(x0, x1, lists[warp + lvl][lane], lists[warp + lvl][lane + 32], lane);
      lists[warp][lane] = x0;
      lists[warp][lane + 32] = x1;
    }
  }
  __syncthreads();
}

// Inclusive prefix sum across the warp's lanes.
__device__ __forceinline__ float warp_scan(float v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

// The first position set in the 64-bit mask (lo: positions 0-31, hi: 32-63), or `none`.
__device__ __forceinline__ int first_set(uint32_t lo, uint32_t hi, int none) {
  if (lo) return __ffs(lo) - 1;
  if (hi) return 32 + __ffs(hi) - 1;
  return none;
}

__device__ __forceinline__ unsigned long long splitmix64(unsigned long long z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Warp 0 of the deciding CTA: from the sorted top keys and the whole
// vocabulary's softmax statistics (max M, sum Z of exp(v - M)), the kept
// positions (i = 0, then up to the first i with cumsum(p)[i] > top_p, at most
// top_k), the softmax of the kept logits / temperature and the inverse-CDF
// draw of one of them.
template <typename Key>
__device__ __forceinline__ void draw_token(const Key* keys, float M, float Z, int V,
                                           float temperature, float top_p, int top_k, unsigned long long seed,
                                           const int64_t* __restrict__ step, int64_t* __restrict__ out, int lane) {
  const int kk = top_k < kTop ? (top_k < 1 ? 1 : top_k) : kTop;
  const int n = kk < V ? kk : V;
  const float inv_t = 1.0f / fmaxf(temperature, 1e-5f);
  const float kv0 = key_value(keys[lane]), kv1 = key_value(keys[lane + 32]);
  const float p0 = lane < n ? expf(kv0 - M) / Z : 0.f, p1 = lane + 32 < n ? expf(kv1 - M) / Z : 0.f;
  const float c0 = warp_scan(p0, lane);
  const float c1 = warp_scan(p1, lane) + __shfl_sync(0xffffffffu, c0, 31);
  const int keep = first_set(__ballot_sync(0xffffffffu, lane >= 1 && lane < n && c0 > top_p),
                             __ballot_sync(0xffffffffu, lane + 32 < n && c1 > top_p), n);
  const float m0 = key_value(keys[0]) * inv_t;
  const float q0 = lane < keep ? expf(kv0 * inv_t - m0) : 0.f;
  const float q1 = lane + 32 < keep ? expf(kv1 * inv_t - m0) : 0.f;
  const float a0 = warp_scan(q0, lane);
  const float a1 = warp_scan(q1, lane) + __shfl_sync(0xffffffffu, a0, 31);
  const float tot = __shfl_sync(0xffffffffu, a1, 31);
  const unsigned long long st = step != nullptr ? (unsigned long long)step[0] : 0ull;
  const float u = (float)(splitmix64(seed ^ (st * 0xD1B54A32D192ED03ull)) >> 40) * (1.0f / 16777216.0f);
  const float target = u * tot;
  const int pick = first_set(__ballot_sync(0xffffffffu, lane < keep && a0 > target),
                             __ballot_sync(0xffffffffu, lane + 32 < keep && a1 > target), keep - 1);
  if (lane == 0) out[0] = (int64_t)key_index(keys[pick]);
}

// `per` slices of 2048 logits per CTA: 1 when the vocabulary takes several
// CTAs, up to kMaxPer for a vocabulary one CTA takes whole (the codebooks'
// 4096), which then draws at once - no partial lists through global memory,
// no last-CTA handoff (a 4096-entry draw took 13.4 us as two CTAs).
constexpr int kMaxPer = 2;
// Key: 32-bit keys for a one-CTA vocabulary, 64-bit otherwise.
template <typename Key>
__global__ void __launch_bounds__(kSThreads) sample_kernel(const uint16_t* __restrict__ logits, int V, int per,
                                                           float temperature, float top_p, int top_k,
                                                           unsigned long long seed, const int64_t* __restrict__ step,
                                                           int64_t* __restrict__ out, unsigned long long* __restrict__ ws_keys,
                                                           float* __restrict__ ws_stats, int* __restrict__ counter) {
  __shared__ Key lists[kSThreads / 32][kTop];
  __shared__ float red_m[kSThreads / 32], red_s[kSThreads / 32];
  __shared__ float sm_max[kMaxSlices], sm_term[kMaxSlices];
  __shared__ int last;
  pdl_wait();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int s = blockIdx.x, S = gridDim.x;
  const int base = s * kSlice * per;
  // this CTA's keys (64 per warp and slice, sorted in registers, the slices'
  // lists merged) and its max / sum of exp
  float v[2 * kMaxPer];
  Key x0 = 0, x1 = 0;  // 0: below every real key
  float m = -INFINITY;
#pragma unroll
  for (int c = 0; c < kMaxPer; ++c) {
    v[2 * c] = v[2 * c + 1] = -INFINITY;
    if (c >= per) continue;
    const int j0 = base + c * kSlice + warp * 64 + lane, j1 = j0 + 32;
    v[2 * c] = j0 < V ? bf2f(logits[j0]) : -INFINITY;
    v[2 * c + 1] = j1 < V ? bf2f(logits[j1]) : -INFINITY;
    Key y0 = j0 < V ? make_key_t<Key>(v[2 * c], (uint32_t)j0) : Key(0);
    Key y1 = j1 < V ? make_key_t<Key>(v[2 * c + 1], (uint32_t)j1) : Key(0);
    m = fmaxf(m, fmaxf(v[2 * c], v[2 * c + 1]));
    warp_sort64(y0, y1, lane);
    if (c == 0) {
      x0 = y0;
      x1 = y1;
    } else {
      warp_merge64(x0, x1, y0, y1, lane);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if (lane == 0) red_m[warp] = m;
  __syncthreads();
  m = -INFINITY;
  for (int w = 0; w < kSThreads / 32; ++w) m = fmaxf(m, red_m[w]);
  float sum = 0.f;
#pragma unroll
  for (int c = 0; c < 2 * kMaxPer; ++c) sum += expf(v[c] - m);  // exp(-inf) = 0 past the vocabulary
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  if (lane == 0) red_s[warp] = sum;
  block_merge(lists, x0, x1, warp, lane);  // its barriers also publish red_s
  if (S == 1) {
    // the whole vocabulary in this CTA: draw now
    if (warp == 0) {
      float t = 0.f;
      for (int w = 0; w < kSThreads / 32; ++w) t += red_s[w];  // fixed order
      draw_token(lists[0], m, t, V, temperature, top_p, top_k, seed, step, out, lane);
    }
    pdl_launch_dependents();
    return;
  }
  if constexpr (sizeof(Key) == 8) {  // several CTAs: partial lists, the last CTA draws
    if (warp == 0) {
      ws_keys[(size_t)s * kTop + lane] = x0;
      ws_keys[(size_t)s * kTop + lane + 32] = x1;
    }
    if (tid == 0) {
      float t = 0.f;
      for (int w = 0; w < kSThreads / 32; ++w) t += red_s[w];  // fixed order
      ws_stats[2 * s] = m;
      ws_stats[2 * s + 1] = t;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const int old = atomicAdd(counter, 1);
      last = (old == S - 1);
      if (last) *counter = 0;
    }
    __syncthreads();
    if (!last) {
      pdl_launch_dependents();
      return;
    }
    __threadfence();
    // ---- the last CTA: global top keys, full-vocabulary softmax statistics, draw
    x0 = x1 = 0ull;
    for (int c = warp; c < S; c += kSThreads / 32) {
      const unsigned long long b0 = __ldcg(ws_keys + (size_t)c * kTop + lane);
      const unsigned long long b1 = __ldcg(ws_keys + (size_t)c * kTop + lane + 32);
      warp_merge64(x0, x1, b0, b1, lane);
    }
    for (int c = tid; c < S; c += kSThreads) sm_max[c] = __ldcg(ws_stats + 2 * c);
    block_merge(lists, x0, x1, warp, lane);  // its barriers also publish sm_max
    if (warp == 0) {
      float M = -INFINITY;
      for (int c = lane; c < S; c += 32) M = fmaxf(M, sm_max[c]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
      for (int c = lane; c < S; c += 32) sm_term[c] = __ldcg(ws_stats + 2 * c + 1) * expf(sm_max[c] - M);
      __syncwarp();
      float Z = 0.f;
      for (int c = 0; c < S; ++c) Z += sm_term[c];  // slice order (every lane, same value)
      draw_token(lists[0], M, Z, V, temperature, top_p, top_k, seed, step, out, lane);
    }
  }
  pdl_launch_dependents();
}

}  // namespace

size_t sampler_workspace_bytes(int V) {
  const int S = (V + kSlice - 1) / kSlice;
  return 256 + (size_t)S * kTop * 8 + (size_t)S * 2 * 4;
}

cudaError_t launch_sampler(const uint16_t* logits, int V, float temperature, float top_p, int top_k,
                           unsigned long long seed, const int64_t* step, int64_t* out, void* workspace,
                           cudaStream_t stream) {
  // a vocabulary of up to kMaxPer slices: one CTA, no handoff
  const int per = V <= kMaxPer * kSlice ? (V + kSlice - 1) / kSlice : 1;
  const int S = V <= kMaxPer * kSlice ? 1 : (V + kSlice - 1) / kSlice;
  int* counter = static_cast<int*>(workspace);
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(workspace) + 256);
  float* stats = reinterpret_cast<float*>(keys + (size_t)S * kTop);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(S);
  cfg.blockDim = dim3(kSThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (S == 1)
    return cudaLaunchKernelEx(&cfg, sample_kernel<uint32_t>, logits, V, per < 1 ? 1 : per, temperature, top_p, top_k,
                              seed, step, out, keys, stats, counter);
  return cudaLaunchKernelEx(&cfg, sample_kernel<unsigned long long>, logits, V, per < 1 ? 1 : per, temperature, top_p,
                            top_k, seed, step, out, keys, stats, counter);
}

}  // namespace nf4b
