// NF4 -> bf16 dequantisation, bit-exact to bitsandbytes' dequantize_4bit
// (code[q] * scale in fp32, rounded to nearest-even bf16; the per-element value
// of app/engine/nf4gemv.py:185-188 in bf16). One thread turns one 32-bit word
// of packed codes (8 weights) into one 16-byte store. Memory-bound; used to
// pin the dequantised values in tests and as a building block for callers that
// want a dense copy.

#include "common.cuh"
#include "kernels.cuh"

namespace nf4b {


namespace {

__global__ void __launch_bounds__(256) nf4_dequant_kernel(const DequantParams p) {
  const long long words = (long long)p.N * p.K / 8;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < words; i += stride) {
    const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(p.packed) + i);
    const long long b = (i * 8) >> p.bs_shift;  // 8 codes never straddle a block
    float s;
    if (p.nested) {
      s = nested_scale(__ldg(p.code2 + __ldg(p.a8 + b)), __ldg(p.absmax + (b >> p.bs2_shift)),
                       p.offset);
    } else {
      s = __ldg(p.absmax + b);
    }
    uint32_t out[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t byte = (w >> (8 * j)) & 0xFFu;
      out[j] = pack_bf16x2(__fmul_rn(c_nf4_code[byte >> 4], s), __fmul_rn(c_nf4_code[byte & 15], s));
    }
    reinterpret_cast<uint4*>(p.out)[i] = make_uint4(out[0], out[1], out[2], out[3]);
  }
}

}  // namespace

cudaError_t launch_dequant(const DequantParams& p, cudaStream_t stream) {
  const long long words = (long long)p.N * p.K / 8;
  long long blocks = (words + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (blocks < 1) blocks = 1;
  nf4_dequant_kernel<<<(unsigned)blocks, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace nf4b
