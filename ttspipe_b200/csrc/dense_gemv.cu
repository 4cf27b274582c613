// Dense bf16 decode GEMV for the output heads (the slow AR's 2560 -> 155136 LM
// head, the fast AR's 2560 -> 4096 codebook heads): y = bf16(x W^T), one
// activation row, fp32 accumulation: the fork's bf16 nn.Linear heads, which the
// reference runs through torch (app/engine/graphs.py:205-217 replays them).
//
// HBM-bound (2 bytes of weight per multiply-add), so no tensor cores: a
// persistent grid of 16-warp CTAs, one weight row per warp at a time, every
// lane reading 16 contiguous bytes per load so a warp's load covers 512
// contiguous bytes of the row. Each warp keeps the next row's loads in flight
// while it reduces the current one (register double buffer); x is staged in
// shared memory (k_in <= 4096), RMS-normalised there first when a norm weight
// is given (nf4b_rms_norm's arithmetic: the fast AR's norm before each
// codebook head, app/engine/graphs.py:205-217).

#include "common.cuh"
#include "kernels.cuh"

namespace nf4b {

namespace {

constexpr int kDWarps = 16;
constexpr int kDThreads = kDWarps * 32;

template <int C>  // 512-byte column chunks per row: k_in = 256 * C
__global__ void __launch_bounds__(kDThreads, 1) dense_gemv_kernel(const uint16_t* __restrict__ w,
                                                                  const uint16_t* __restrict__ x,
                                                                  uint16_t* __restrict__ y, int n_out,
                                                                  const uint16_t* __restrict__ norm_w,
                                                                  float norm_eps) {
  __shared__ __align__(16) uint4 xs[C * 32];
  __shared__ double red[kDWarps];
  const int lane = threadIdx.x & 31;
  const long long gw = (long long)blockIdx.x * kDWarps + (threadIdx.x >> 5);
  const long long W = (long long)gridDim.x * kDWarps;
  constexpr int K = 256 * C;
  // Weight rows are static: the first row's loads go out before the wait for
  // the previous kernel (x and y belong to the stream's earlier work).
  uint4 cur[C], nxt[C];
  long long r = gw;
  if (r < n_out) {
    const uint4* src = reinterpret_cast<const uint4*>(w + r * K) + lane;
#pragma unroll
    for (int c = 0; c < C; ++c) cur[c] = ld_stream_u4(src + c * 32);
  }
  pdl_wait();
  for (int i = threadIdx.x; i < C * 32; i += kDThreads) xs[i] = reinterpret_cast<const uint4*>(x)[i];
  __syncthreads();
  if (norm_w != nullptr) rms_normalise_staged<kDThreads>(reinterpret_cast<uint16_t*>(xs), 1, K, norm_w, norm_eps, red);
  pdl_launch_dependents();
  for (; r < n_out; r += W) {
    const long long rn = r + W;
    if (rn < n_out) {
      const uint4* src = reinterpret_cast<const uint4*>(w + rn * K) + lane;
#pragma unroll
      for (int c = 0; c < C; ++c) nxt[c] = ld_stream_u4(src + c * 32);
    }
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const uint4 wv = cur[c], xv = xs[c * 32 + lane];
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w}, xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        acc = fmaf(__uint_as_float(ww[e] << 16), __uint_as_float(xx[e] << 16), acc);
        acc = fmaf(__uint_as_float(ww[e] & 0xFFFF0000u), __uint_as_float(xx[e] & 0xFFFF0000u), acc);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) y[r] = f2bf(acc);
#pragma unroll
    for (int c = 0; c < C; ++c) cur[c] = nxt[c];
  }
}

template <int C>
cudaError_t launch_c(const uint16_t* w, const uint16_t* x, uint16_t* y, int n_out, int sms, const uint16_t* norm_w,
                     float norm_eps, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  long long ctas = ((long long)n_out + kDWarps - 1) / kDWarps;
  if (ctas > sms) ctas = sms;
  cfg.gridDim = dim3((unsigned)ctas);
  cfg.blockDim = dim3(kDThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, dense_gemv_kernel<C>, w, x, y, n_out, norm_w, norm_eps);
}

}  // namespace

cudaError_t launch_dense_gemv(const uint16_t* w, const uint16_t* x, uint16_t* y, int n_out, int k_in, int sms,
                              const uint16_t* norm_w, float norm_eps, cudaStream_t stream) {
  switch (k_in / 256) {
    case 4: return launch_c<4>(w, x, y, n_out, sms, norm_w, norm_eps, stream);
    case 8: return launch_c<8>(w, x, y, n_out, sms, norm_w, norm_eps, stream);
    case 10: return launch_c<10>(w, x, y, n_out, sms, norm_w, norm_eps, stream);
    case 16: return launch_c<16>(w, x, y, n_out, sms, norm_w, norm_eps, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace nf4b
