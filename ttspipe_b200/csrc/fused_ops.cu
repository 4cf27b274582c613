// RMSNorm, rotary embedding and the decode-step q/k norm + rotary + KV write.
//
// Same formulas and rounding points as the reference kernels
// (app/engine/fusedops.py:61-132, app/engine/fusedlayer.py:56-92) with bf16
// activations, or fp16 (F16) as the reference's own kernels. The sum of squares is accumulated in fp64: every term is an
// exact square of a bf16 / fp16 value, so the sum is exact in any order and the norm
// does not depend on the reduction tree; the reciprocal square root is the
// correctly rounded fp32 value. Rotary is spelled with the _rn intrinsics so
// no multiply-add is contracted: (x0*c - x1*s, x1*c + x0*s), each product and
// the sum rounded in fp32.

#include "common.cuh"
#include "kernels.cuh"

namespace nf4b {

namespace {

template <int THREADS>
__device__ __forceinline__ double block_sum(double v, double* red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  constexpr int WARPS = THREADS / 32;
  if (WARPS == 1) return v;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double s = 0.0;
#pragma unroll
  for (int i = 0; i < WARPS; ++i) s += red[i];
  return s;
}

constexpr int kNormThreads = 256;

template <bool F16>
__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(const bf16_t* __restrict__ x,
                                                                const bf16_t* __restrict__ w,
                                                                bf16_t* __restrict__ y, int width,
                                                                float eps) {
  __shared__ double red[kNormThreads / 32];
  pdl_wait();
  const size_t base = (size_t)blockIdx.x * width;
  double ss = 0.0;
  for (int i = threadIdx.x; i < width; i += kNormThreads) {
    const double v = act2f<F16>(x[base + i]);
    ss += v * v;
  }
  ss = block_sum<kNormThreads>(ss, red);
  const float r = rsqrt_exact(ss, width, eps);
  for (int i = threadIdx.x; i < width; i += kNormThreads) {
    const float normed = round_act<F16>(__fmul_rn(act2f<F16>(x[base + i]), r));
    y[base + i] = f2act<F16>(__fmul_rn(normed, act2f<F16>(w[i])));
  }
  pdl_launch_dependents();
}

template <bool F16>
__global__ void __launch_bounds__(256) rope_kernel(const bf16_t* __restrict__ x,
                                                   const void* __restrict__ f, int ftype,
                                                   bf16_t* __restrict__ y, long long pairs,
                                                   int half_dim, int heads, int seq) {
  pdl_wait();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < pairs) {
    const int p = (int)(i % half_dim);
    const long long s = (i / half_dim / heads) % seq;
    const long long fi = (s * half_dim + p) * 2;
    const float c = load_freq(f, fi, ftype), sn = load_freq(f, fi + 1, ftype);
    const float x0 = act2f<F16>(x[2 * i]), x1 = act2f<F16>(x[2 * i + 1]);
    y[2 * i] = f2act<F16>(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)));
    y[2 * i + 1] = f2act<F16>(__fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, sn)));
  }
  pdl_launch_dependents();
}

// One CTA per head (n_head query heads, then n_kv key heads, then n_kv value
// heads), one thread per dimension of a 128-wide head.
constexpr int kHeadDim = 128;

template <bool F16>
__global__ void __launch_bounds__(kHeadDim) qk_rope_kv_kernel(
    const bf16_t* __restrict__ qkv, const bf16_t* __restrict__ qw, const bf16_t* __restrict__ kw,
    float eps, const void* __restrict__ f, int ftype, const int64_t* __restrict__ pos_ptr,
    bf16_t* __restrict__ q_out, bf16_t* __restrict__ kc, bf16_t* __restrict__ vc, int nh, int nkv,
    int max_len) {
  __shared__ float sx[kHeadDim];
  __shared__ double red[kHeadDim / 32];
  pdl_wait();
  const int head = blockIdx.x, d = threadIdx.x;
  const long long pos = pos_ptr[0];
  if (head >= nh + nkv) {
    const int vh = head - nh - nkv;
    vc[((size_t)vh * max_len + pos) * kHeadDim + d] = qkv[(size_t)(nh + nkv + vh) * kHeadDim + d];
    pdl_launch_dependents();
    return;
  }
  const bool is_q = head < nh;
  float x = act2f<F16>(qkv[(size_t)head * kHeadDim + d]);
  const bf16_t* w = is_q ? qw : kw;
  if (w != nullptr) {
    const double sq = (double)x * (double)x;
    const double ss = block_sum<kHeadDim>(sq, red);
    const float r = rsqrt_exact(ss, kHeadDim, eps);
    x = round_act<F16>(__fmul_rn(__fmul_rn(x, r), act2f<F16>(w[d])));
  }
  sx[d] = x;
  __syncthreads();
  const float x0 = sx[d & ~1], x1 = sx[d | 1];
  const float c = load_freq(f, d & ~1, ftype), sn = load_freq(f, d | 1, ftype);
  const float r = (d & 1) ? __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, sn))
                          : __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
  if (is_q)
    q_out[(size_t)head * kHeadDim + d] = f2act<F16>(r);
  else
    kc[((size_t)(head - nh) * max_len + pos) * kHeadDim + d] = f2act<F16>(r);
  pdl_launch_dependents();
}

cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, void** args, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace

cudaError_t launch_rms_norm(const uint16_t* x, const uint16_t* w, uint16_t* y, int rows,
                            int width, float eps, cudaStream_t stream, bool f16) {
  void* args[] = {(void*)&x, (void*)&w, (void*)&y, (void*)&width, (void*)&eps};
  return launch_pdl(f16 ? (const void*)rms_norm_kernel<true> : (const void*)rms_norm_kernel<false>, dim3(rows),
                    dim3(kNormThreads), args, stream);
}

cudaError_t launch_rope(const uint16_t* x, const void* freqs, int ftype, uint16_t* y,
                        long long pairs, int half_dim, int heads, int seq, cudaStream_t stream, bool f16) {
  const long long blocks = (pairs + 255) / 256;
  void* args[] = {(void*)&x, (void*)&freqs, (void*)&ftype, (void*)&y,
                  (void*)&pairs, (void*)&half_dim, (void*)&heads, (void*)&seq};
  return launch_pdl(f16 ? (const void*)rope_kernel<true> : (const void*)rope_kernel<false>, dim3((unsigned)blocks),
                    dim3(256), args, stream);
}

cudaError_t launch_qk_rope_kv(const uint16_t* qkv, const uint16_t* qw, const uint16_t* kw,
                              float eps, const void* freqs, int ftype, const int64_t* pos,
                              uint16_t* q_out, uint16_t* kc, uint16_t* vc, int nh, int nkv,
                              int max_len, cudaStream_t stream, bool f16) {
  void* args[] = {(void*)&qkv, (void*)&qw, (void*)&kw, (void*)&eps, (void*)&freqs,
                  (void*)&ftype, (void*)&pos, (void*)&q_out, (void*)&kc, (void*)&vc,
                  (void*)&nh, (void*)&nkv, (void*)&max_len};
  return launch_pdl(f16 ? (const void*)qk_rope_kv_kernel<true> : (const void*)qk_rope_kv_kernel<false>,
                    dim3(nh + 2 * nkv), dim3(kHeadDim), args, stream);
}

}  // namespace nf4b
