// Shared device helpers for the sm_100a NF4 hot-path kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "nf4b200.h"

namespace nf4b {

typedef uint16_t bf16_t;  // bf16 bit pattern; arithmetic is always fp32

// bitsandbytes' NF4 code points in index order (app/engine/nf4gemv.py:69-86).
static __constant__ float c_nf4_code[16] = {
    -1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
    -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
    0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f, 0.33791524171829224f,
    0.44070982933044434f, 0.5626170039176941f, 0.7229568362236023f, 1.0f};

__device__ __forceinline__ float bf2f(bf16_t b) { return __uint_as_float(((uint32_t)b) << 16); }

// Round to nearest even; NaN stays NaN (cvt handles it).
__device__ __forceinline__ bf16_t f2bf(float f) {
  uint16_t r;
  asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r) : "f"(f));
  return r;
}

__device__ __forceinline__ float round_bf(float f) { return bf2f(f2bf(f)); }

// fp16 (binary16) bit patterns, for the fp16 activations the reference serves
// by default: widening is exact, narrowing rounds to nearest even (cvt.rn),
// overflow goes to infinity as in torch.
__device__ __forceinline__ float h2f(uint16_t h) {
  float f;
  asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h));
  return f;
}
__device__ __forceinline__ uint16_t f2h(float f) {
  uint16_t h;
  asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(f));
  return h;
}

// The activation type of a kernel instantiation: bf16 (F16 = false) or fp16.
template <bool F16>
__device__ __forceinline__ float act2f(uint16_t v) {
  return F16 ? h2f(v) : bf2f(v);
}
template <bool F16>
__device__ __forceinline__ uint16_t f2act(float f) {
  return F16 ? f2h(f) : f2bf(f);
}
template <bool F16>
__device__ __forceinline__ float round_act(float f) {
  return act2f<F16>(f2act<F16>(f));
}

// The low / high 16-bit value of a packed pair of the activation type, widened
// (exact). For bf16 a shift or a mask is the whole conversion.
template <bool F16>
__device__ __forceinline__ float act_lo(uint32_t w) {
  return F16 ? h2f((uint16_t)(w & 0xFFFFu)) : __uint_as_float(w << 16);
}
template <bool F16>
__device__ __forceinline__ float act_hi(uint32_t w) {
  return F16 ? h2f((uint16_t)(w >> 16)) : __uint_as_float(w & 0xFFFF0000u);
}

// Two fp32 -> one bf16x2 register, `lo` in the low half (lower address).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
template <bool F16>
__device__ __forceinline__ uint32_t pack_act2(float lo, float hi) {
  return F16 ? pack_f16x2(lo, hi) : pack_bf16x2(lo, hi);
}

// Streaming read of data used once (packed weights): no L1 allocation, and a
// 256-byte L2 prefetch so the neighbouring sectors of the row arrive with it.
__device__ __forceinline__ uint2 ld_stream_u2(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v2.u32 {%0, %1}, [%2];"
               : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}


// Programmatic dependent launch: let the next kernel in the stream start its
// prologue, and wait for the previous kernel's results before reading them.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// The per-block scale of a bitsandbytes NF4 weight: plain fp32 absmax, or the
// doubly quantised code2[a8] * absmax2 + offset as two separately rounded
// fp32 operations (the reconstruction bitsandbytes and the reference do).
__device__ __forceinline__ float nested_scale(float code2_val, float absmax2_val, float offset) {
  return __fadd_rn(__fmul_rn(code2_val, absmax2_val), offset);
}

// One 64-block's dequantisation table: entry i = RNE_bf16(NF4[i] * scale) (the
// fp32 product, so bit-exact), stored as byte planes - lo[j] holds the low
// bytes of entries 4j..4j+3, hi[j] their high bytes - so that byte permutes
// can look entries up without memory.
struct ScaledLut {
  uint32_t lo[4], hi[4];
};

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

template <bool F16 = false>
__device__ __forceinline__ ScaledLut scaled_lut(float scale) {
  uint32_t pair[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    pair[i] = pack_act2<F16>(__fmul_rn(c_nf4_code[2 * i], scale), __fmul_rn(c_nf4_code[2 * i + 1], scale));
  ScaledLut t;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    t.lo[j] = prmt(pair[2 * j], pair[2 * j + 1], 0x6420u);
    t.hi[j] = prmt(pair[2 * j], pair[2 * j + 1], 0x7531u);
  }
  return t;
}

// Dequantise one 32-bit word of packed codes (8 weights, byte j = codes 2j
// (high nibble) and 2j+1) into four bf16x2 words in k order. Per nibble: a
// 3-bit permute into each half of the table, a select on the nibble's top
// bit (a mask made with the permute's sign-replicating mode), then the low
// and high byte planes are interleaved back into bf16 values.
__device__ __forceinline__ void lut_dequant8(const ScaledLut& t, uint32_t w, uint32_t (&o)[4]) {
  const uint32_t w4 = w << 4;
  const uint32_t m_lo = prmt(w4, w, 0xD9C8u), m_hi = prmt(w4, w, 0xFBEAu);
  const uint32_t s_lo = w & 0x7777u, s_hi = (w >> 16) & 0x7777u;
  uint32_t l = (prmt(t.lo[0], t.lo[1], s_lo) & ~m_lo) | (prmt(t.lo[2], t.lo[3], s_lo) & m_lo);
  uint32_t h = (prmt(t.hi[0], t.hi[1], s_lo) & ~m_lo) | (prmt(t.hi[2], t.hi[3], s_lo) & m_lo);
  o[0] = prmt(l, h, 0x4051u);
  o[1] = prmt(l, h, 0x6273u);
  l = (prmt(t.lo[0], t.lo[1], s_hi) & ~m_hi) | (prmt(t.lo[2], t.lo[3], s_hi) & m_hi);
  h = (prmt(t.hi[0], t.hi[1], s_hi) & ~m_hi) | (prmt(t.hi[2], t.hi[3], s_hi) & m_hi);
  o[2] = prmt(l, h, 0x4051u);
  o[3] = prmt(l, h, 0x6273u);
}

// Epilogue applied to one fp32 accumulator: the matmul output is rounded to
// bf16 first, then the fused op rounds again where the unfused model does.
// Element i of a rotary table of dtype NF4B_F32 / NF4B_F16 / NF4B_BF16.
__device__ __forceinline__ float load_freq(const void* f, long long i, int ftype) {
  if (ftype == NF4B_F32) return reinterpret_cast<const float*>(f)[i];
  if (ftype == NF4B_F16) return __half2float(reinterpret_cast<const __half*>(f)[i]);
  return bf2f(reinterpret_cast<const bf16_t*>(f)[i]);
}

// RMSNorm's scale from an fp64 sum of squares: the correctly rounded fp32
// 1 / sqrt(fp32(ss / width) + eps).
__device__ __forceinline__ float rsqrt_exact(double ss, int width, float eps) {
  const float t = __fadd_rn((float)(ss / (double)width), eps);
  return (float)(1.0 / sqrt((double)t));
}

// RMS-normalise the M rows of K bf16 values staged at xr (shared memory) in
// place with weight w, with the arithmetic of nf4b_rms_norm: fp64 sum of
// squares (exact for bf16 inputs, so its order does not matter),
// r = 1 / sqrt(fp32(ss / K) + eps), y = bf16(bf16(x * r) * w). Called by every
// thread of the CTA after a barrier that made x visible; ends with a barrier.
// `red` holds one double per warp. Row m starts at element m * row_stride
// (K for kLayout 0). kLayout 0: contiguous; 1: every 64 elements are followed
// by 8 elements of padding; 2: each 64-element block's eight 8-element chunks
// are rotated, chunk c of block b at chunk (c + (b & 3) + 4 (m & 1)) & 7.
template <int THREADS, int kLayout = 0, bool F16 = false>
__device__ __forceinline__ void rms_normalise_staged(uint16_t* xr, int M, int K, const uint16_t* __restrict__ w,
                                                     float eps, double* red, int row_stride = 0) {
  constexpr int NW = THREADS / 32;
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int rs = kLayout ? row_stride : K;
  auto at = [&](int m, int i) -> uint16_t& {
    if (kLayout == 1) return xr[m * rs + i + ((i >> 6) << 3)];
    if (kLayout == 2) {
      const int b = i >> 6, c = (((i >> 3) & 7) + (b & 3) + 4 * (m & 1)) & 7;
      return xr[m * rs + (b << 6) + (c << 3) + (i & 7)];
    }
    return xr[m * rs + i];
  };
  for (int m = 0; m < M; ++m) {
    double ss = 0.0;
    for (int i = threadIdx.x; i < K; i += THREADS) {
      const double v = act2f<F16>(at(m, i));
      ss += v * v;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) red[wib] = ss;
    __syncthreads();
    double tot = 0.0;
#pragma unroll
    for (int k = 0; k < NW; ++k) tot += red[k];
    const float r = rsqrt_exact(tot, K, eps);
    for (int i = threadIdx.x; i < K; i += THREADS) {
      const float normed = round_act<F16>(__fmul_rn(act2f<F16>(at(m, i)), r));
      at(m, i) = f2act<F16>(__fmul_rn(normed, act2f<F16>(__ldg(w + i))));
    }
    __syncthreads();
  }
}

// The epilogue with the operand value already loaded (ignored for NF4B_EPI_NONE),
// at the activation type's rounding points.
template <bool F16 = false>
__device__ __forceinline__ uint16_t epilogue_value(float acc, int epi, float opv) {
  const float y = round_act<F16>(acc);
  if (epi == NF4B_EPI_RESIDUAL) {
    return f2act<F16>(__fadd_rn(opv, y));
  } else if (epi == NF4B_EPI_SILU_GATE) {
    const float s = round_act<F16>(__fdiv_rn(opv, __fadd_rn(1.0f, expf(-opv))));
    return f2act<F16>(__fmul_rn(s, y));
  }
  return f2act<F16>(y);
}

template <bool F16 = false>
__device__ __forceinline__ uint16_t epilogue(float acc, int epi, const uint16_t* operand, size_t idx) {
  return epilogue_value<F16>(acc, epi, epi == NF4B_EPI_NONE ? 0.f : act2f<F16>(operand[idx]));
}

}  // namespace nf4b
