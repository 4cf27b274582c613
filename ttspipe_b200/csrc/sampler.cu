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
// One launch. CTA s sorts a 2048-logit slice (bitonic network on 64-bit
// (value, index) keys: larger value first, then smaller index), publishes its
// 64 best keys and its (max, sum of exp) for the full-vocabulary softmax; the
// last CTA (atomic counter, reset after use) sorts the slices' winners and
// draws. The draw is inverse-CDF with one uniform from a counter-based hash
// of (seed, *step) - the same distribution as the fork's exponential race,
// reproducible from the seed.

#include "common.cuh"
#include "kernels.cuh"

namespace nf4b {

namespace {

constexpr int kSlice = 2048;
constexpr int kSThreads = 1024;
constexpr int kTop = 64;

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

// Descending bitonic sort of n (power of two) keys in shared memory.
__device__ void bitonic_desc(unsigned long long* a, int n) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int i = threadIdx.x; i < n / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool desc = ((lo & size) == 0);
        const unsigned long long x = a[lo], y = a[hi];
        if ((x < y) == desc) {
          a[lo] = y;
          a[hi] = x;
        }
      }
    }
  }
  __syncthreads();
}

__device__ __forceinline__ unsigned long long splitmix64(unsigned long long z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void __launch_bounds__(kSThreads) sample_kernel(const uint16_t* __restrict__ logits, int V,
                                                           float temperature, float top_p, int top_k,
                                                           unsigned long long seed, const int64_t* __restrict__ step,
                                                           int64_t* __restrict__ out, unsigned long long* __restrict__ ws_keys,
                                                           float* __restrict__ ws_stats, int* __restrict__ counter) {
  extern __shared__ __align__(16) unsigned long long keys[];
  __shared__ float red_m[kSThreads / 32], red_s[kSThreads / 32];
  __shared__ int last;
  pdl_wait();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int s = blockIdx.x, S = gridDim.x;
  const int base = s * kSlice;
  // this slice's keys and its max / sum of exp
  float m = -INFINITY;
  for (int i = tid; i < kSlice; i += kSThreads) {
    const int j = base + i;
    if (j < V) {
      const float v = bf2f(logits[j]);
      keys[i] = make_key(v, (uint32_t)j);
      m = fmaxf(m, v);
    } else {
      keys[i] = 0ull;  // below every real key
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if (lane == 0) red_m[warp] = m;
  __syncthreads();
  m = -INFINITY;
  for (int w = 0; w < kSThreads / 32; ++w) m = fmaxf(m, red_m[w]);
  float sum = 0.f;
  for (int i = tid; i < kSlice; i += kSThreads) {
    const int j = base + i;
    if (j < V) sum += expf(bf2f(logits[j]) - m);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  if (lane == 0) red_s[warp] = sum;
  bitonic_desc(keys, kSlice);
  if (tid < kTop) ws_keys[(size_t)s * kTop + tid] = keys[tid];
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
  int P = kTop;
  while (P < S * kTop) P <<= 1;
  for (int i = tid; i < P; i += kSThreads) keys[i] = i < S * kTop ? __ldcg(ws_keys + i) : 0ull;
  bitonic_desc(keys, P);
  if (tid == 0) {
    float M = -INFINITY;
    for (int c = 0; c < S; ++c) M = fmaxf(M, __ldcg(ws_stats + 2 * c));
    float Z = 0.f;
    for (int c = 0; c < S; ++c) Z += __ldcg(ws_stats + 2 * c + 1) * expf(__ldcg(ws_stats + 2 * c) - M);
    const int kk = top_k < kTop ? (top_k < 1 ? 1 : top_k) : kTop;
    const int n = kk < V ? kk : V;
    const float inv_t = 1.0f / fmaxf(temperature, 1e-5f);
    // kept positions: a prefix of the sorted list (cumsum is increasing)
    float cum = 0.f;
    int keep = 0;
    for (int i = 0; i < n; ++i) {
      cum += expf(key_value(keys[i]) - M) / Z;
      if (i > 0 && cum > top_p) break;
      keep = i + 1;
    }
    // softmax of the kept logits / temperature, then the inverse-CDF draw
    const float m0 = key_value(keys[0]) * inv_t;
    float tot = 0.f;
    for (int i = 0; i < keep; ++i) tot += expf(key_value(keys[i]) * inv_t - m0);
    const unsigned long long st = step != nullptr ? (unsigned long long)step[0] : 0ull;
    const float u = (float)(splitmix64(seed ^ (st * 0xD1B54A32D192ED03ull)) >> 40) * (1.0f / 16777216.0f);
    const float target = u * tot;
    float acc = 0.f;
    int pick = keep - 1;
    for (int i = 0; i < keep; ++i) {
      acc += expf(key_value(keys[i]) * inv_t - m0);
      if (acc > target) {
        pick = i;
        break;
      }
    }
    out[0] = (int64_t)key_index(keys[pick]);
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
  const int S = (V + kSlice - 1) / kSlice;
  int P = kTop;
  while (P < S * kTop) P <<= 1;
  const int smem = (P > kSlice ? P : kSlice) * 8;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  int* counter = static_cast<int*>(workspace);
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(workspace) + 256);
  float* stats = reinterpret_cast<float*>(keys + (size_t)S * kTop);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(S);
  cfg.blockDim = dim3(kSThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, sample_kernel, logits, V, temperature, top_p, top_k, seed, step, out, keys, stats,
                            counter);
}

}  // namespace nf4b
