// Device helpers shared by the register-fed NF4 GEMV kernels (nf4_gemv.cu)
// and the persistent decode-step kernel (decode_step.cu): the NF4 pair table,
// the code2 copies, the bf16 MMA, the 256-bit weight loads and the FeedForward
// gate's rounding points.
#pragma once

#include "common.cuh"

namespace nf4b {
namespace {

__device__ __forceinline__ uint32_t lut_lookup(const uint8_t* lut, uint32_t word, uint32_t sel,
                                               uint32_t lane_base) {
  // Byte permute: {lane_base.b0, word.b[j], 0, 0} = entry * 256 + lane * 4.
  const uint32_t off = __byte_perm(word, lane_base, sel);
  return *reinterpret_cast<const uint32_t*>(lut + off);
}

// Selector that picks byte j of the word (see lut_lookup).
__host__ __device__ constexpr uint32_t lut_sel(int j) { return 0x5504u | ((uint32_t)j << 4); }

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1,
                                              uint32_t a2, uint32_t a3, uint32_t b0,
                                              uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// The MMA of the activation type (both operands of one type, as kind::f16 requires).
template <bool F16>
__device__ __forceinline__ void mma_act(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  if (F16)
    mma_f16_16816(d, a0, a1, a2, a3, b0, b1);
  else
    mma_bf16_16816(d, a0, a1, a2, a3, b0, b1);
}


// NF4 code point q (0..15) from immediates (a select tree): the tables below
// are built without a constant-bank load, which misses in a fresh launch.
__device__ __forceinline__ float nf4_code_imm(uint32_t q) {
  const bool b0 = q & 1u, b1 = q & 2u, b2 = q & 4u, b3 = q & 8u;
  const float l0 = b0 ? -0.6961928009986877f : -1.0f;
  const float l1 = b0 ? -0.39491748809814453f : -0.5250730514526367f;
  const float l2 = b0 ? -0.18477343022823334f : -0.28444138169288635f;
  const float l3 = b0 ? 0.0f : -0.09105003625154495f;
  const float l4 = b0 ? 0.16093020141124725f : 0.07958029955625534f;
  const float l5 = b0 ? 0.33791524171829224f : 0.24611230194568634f;
  const float l6 = b0 ? 0.5626170039176941f : 0.44070982933044434f;
  const float l7 = b0 ? 1.0f : 0.7229568362236023f;
  const float m0 = b1 ? l1 : l0, m1 = b1 ? l3 : l2, m2 = b1 ? l5 : l4, m3 = b1 ? l7 : l6;
  const float n0 = b2 ? m1 : m0, n1 = b2 ? m3 : m2;
  return b3 ? n1 : n0;
}


// The pair table with conflict-free stores: the 8 threads of a quarter warp
// write the 8 16-byte pieces of one entry (128 contiguous bytes); the 16 code
// values come from lanes 0..15 by shuffle. Called by whole warps. Entries are
// code pairs of the activation type (F16: fp16, else bf16).
template <int THREADS, bool F16 = false>
__device__ __forceinline__ void build_pair_lut_fast(uint8_t* smem) {
  const float code = nf4_code_imm((uint32_t)(threadIdx.x & 15));
#pragma unroll
  for (int r = 0; r < 2048 / THREADS; ++r) {
    const int idx = threadIdx.x + r * THREADS, e = idx >> 3, c = idx & 7;
    const float hi_nib = __shfl_sync(0xffffffffu, code, e >> 4);
    const float lo_nib = __shfl_sync(0xffffffffu, code, e & 15);
    const uint32_t v = pack_act2<F16>(hi_nib, lo_nib);
    *reinterpret_cast<uint4*>(smem + e * 256 + c * 16) = make_uint4(v, v, v, v);
  }
}

// The code2 copies of the register-fed kernels, stored conflict-free: entry
// e's 128 bytes at e * 256 + 128 hold 16 copies of code2[e] (W), then 16 of
// code2_3[e] (W3; W's again when there is no W3). `vals` are this thread's
// values, loaded by load_code2_copies.
template <int THREADS>
__device__ __forceinline__ void load_code2_copies(const float* c2, const float* c2_3, float (&vals)[2048 / THREADS]) {
#pragma unroll
  for (int r = 0; r < 2048 / THREADS; ++r) {
    const int idx = threadIdx.x + r * THREADS, e = idx >> 3, c = idx & 7;
    vals[r] = __ldg(((c >= 4 && c2_3 != nullptr) ? c2_3 : c2) + e);
  }
}
template <int THREADS>
__device__ __forceinline__ void store_code2_copies(uint8_t* smem, const float (&vals)[2048 / THREADS]) {
#pragma unroll
  for (int r = 0; r < 2048 / THREADS; ++r) {
    const int idx = threadIdx.x + r * THREADS, e = idx >> 3, c = idx & 7;
    *reinterpret_cast<float4*>(smem + e * 256 + 128 + c * 16) = make_float4(vals[r], vals[r], vals[r], vals[r]);
  }
}


// The gate of a W1/W3 pair at the fork's rounding points:
// bf16(bf16(silu(bf16(x W1))) * bf16(x W3)) (app/engine/fusedlayer.py:265-266).
template <bool F16 = false>
__device__ __forceinline__ uint16_t gate_bf16(float v1, float v3) {
  const float a = round_act<F16>(v1);
  const float s = round_act<F16>(__fdiv_rn(a, __fadd_rn(1.0f, expf(-a))));
  return f2act<F16>(__fmul_rn(s, round_act<F16>(v3)));
}


__device__ __forceinline__ unsigned long long gemv_globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

constexpr int kRegDepth = 3;  // units in flight per warp

__host__ __device__ constexpr int reg_x_row_bytes(int K) { return K * 9 / 4 + 64; }

struct RegSlot {
  uint32_t wa[8], wb[8];  // block t of the unit, rows g and g + 8
  uint32_t qa, qb;        // nested: the unit's four scale codes of rows g, g + 8; plain: block 2(t & 1)'s scale
  uint32_t sa, sb;        // nested: the rows' second-level scale; plain: block 2(t & 1) + 1's scale
};

__device__ __forceinline__ void ld_stream_u8(const void* p, uint32_t (&v)[8]) {
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "l"(p));
}


}  // namespace
}  // namespace nf4b
