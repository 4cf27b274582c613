// Streaming NF4 GEMV for decode (1..32 activation rows) on sm_100a.
//
// Replaces the reference's `nf4_mma` kernel for N <= 32 inputs
// (app/engine/nf4gemv.py:108-231, launch configs :234-248).
//
// Work decomposition. A "unit" is 16 weight rows x one 64-wide k block. Units
// are numbered row-tile-major and split into equal contiguous runs, one run
// per warp of a persistent grid sized to the SM count, so every SM streams the
// same number of bytes whatever the weight shape. A warp that owns a whole row
// tile stores its outputs directly; tiles split between warps are reduced
// through a workspace: each contributor writes its fp32 partial into its own
// slot, and the last to arrive (an atomic counter per tile) sums the slots in
// slot order - deterministic - applies the epilogue and re-zeroes the counter.
//
// Inner loop, per warp and unit: each lane loads 8 packed bytes of two rows
// (g and g+8; the four lanes of a group cover the block's 32 bytes), turns every
// byte into a bf16x2 pair of NF4 code values with one shared-memory lookup
// (a 256-entry pair table, one copy per lane so all 32 lanes hit different
// banks; the address is built with a single byte-permute), and feeds the pairs
// as the A fragment of mma.m16n8k16 with x as B. The block's scale multiplies
// the block's fp32 partial afterwards: y = sum_b s_b * sum_k code[q_k] x_k,
// the factorisation the reference's CPU kernel uses (app/engine/nf4cpu.py:104-131).
// Weights are read with 256-byte L2 prefetch and no L1 allocation, PREFETCH
// units ahead; x is read through L1.
//
// Programmatic dependent launch: the prologue (tables, first weight loads)
// runs before `griddepcontrol.wait`, overlapping the previous kernel's tail;
// nothing the previous kernel writes (x, the workspace, y) is touched before it.

#include "common.cuh"
#include "kernels.cuh"

namespace nf4b {

namespace {

constexpr int kWarps = GEMV_WARPS;
constexpr int kThreads = kWarps * 32;

__device__ __forceinline__ uint32_t lut_lookup(const uint8_t* lut, uint32_t word, uint32_t sel,
                                               uint32_t lane_base) {
  // Byte permute: result = {lane_base.b0, word.b[j], 0, 0} -> entry * 256 + lane * 4.
  const uint32_t off = __byte_perm(word, lane_base, sel);
  return *reinterpret_cast<const uint32_t*>(lut + off);
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct Slot {
  uint2 wa, wb;     // 8 packed bytes of rows g and g+8
  float sa, sb;     // plain: the absmax; nested: absmax2
  uint32_t qa, qb;  // nested: the 8-bit scale codes
};

__device__ __forceinline__ long long warp_of(long long u, long long U, long long W) {
  return ((u + 1) * W - 1) / U;
}

template <int NT>
__global__ void __launch_bounds__(kThreads, 2) nf4_gemv_kernel(const GemvParams p) {
  constexpr int P = (NT == 1) ? 4 : 2;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* lut = smem;
  float* code2_s = reinterpret_cast<float*>(smem + GEMV_LUT_BYTES);

  for (int i = threadIdx.x; i < 256 * 32; i += kThreads) {
    const int e = i >> 5, l = i & 31;
    reinterpret_cast<uint32_t*>(lut)[e * 64 + l] =
        pack_bf16x2(c_nf4_code[e >> 4], c_nf4_code[e & 15]);
  }
  if (p.nested)
    for (int i = threadIdx.x; i < 256; i += kThreads) code2_s[i] = p.code2[i];
  __syncthreads();
  pdl_launch_dependents();

  const int lane = threadIdx.x & 31;
  const long long gw = (long long)blockIdx.x * kWarps + (threadIdx.x >> 5);
  const long long U = p.units, W = p.warps_total;
  if (gw >= W) {
    pdl_wait();
    return;
  }
  const long long u0 = gw * U / W, u1 = (gw + 1) * U / W;
  const int g = lane >> 2, t = lane & 3;
  const int B = p.blocks_per_tile;
  const int N = p.N, K = p.K, M = p.M;
  const size_t row_bytes = (size_t)K >> 1;
  const uint32_t lane_base = (uint32_t)lane * 4u;

  Slot ring[P];
  auto load = [&](long long u, Slot& s) {
    const long long rt = u / B;
    const int kb = (int)(u - rt * B);
    const int ra = min((int)(rt * 16) + g, N - 1), rb = min((int)(rt * 16) + g + 8, N - 1);
    s.wa = ld_stream_u2(p.packed + (size_t)ra * row_bytes + kb * 32 + t * 8);
    s.wb = ld_stream_u2(p.packed + (size_t)rb * row_bytes + kb * 32 + t * 8);
    const size_t ba = ((size_t)ra * K + (size_t)kb * 64) >> p.bs_shift;
    const size_t bb = ((size_t)rb * K + (size_t)kb * 64) >> p.bs_shift;
    if (p.nested) {
      s.qa = __ldg(p.a8 + ba);
      s.qb = __ldg(p.a8 + bb);
      s.sa = __ldg(p.absmax + (ba >> p.bs2_shift));
      s.sb = __ldg(p.absmax + (bb >> p.bs2_shift));
    } else {
      s.sa = __ldg(p.absmax + ba);
      s.sb = __ldg(p.absmax + bb);
    }
  };

#pragma unroll
  for (int i = 0; i < P; ++i)
    if (u0 + i < u1) load(u0 + i, ring[i]);

  pdl_wait();  // x, the workspace and y belong to the stream's previous work

  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;

  auto flush = [&](long long rt) {
    const long long t0 = rt * B, t1 = t0 + B - 1;
    const bool whole = (t0 >= u0) && (t1 < u1);
    int n_contrib = 1, last = 1;
    if (!whole) {
      const long long w_lo = warp_of(t0, U, W);
      n_contrib = (int)(warp_of(t1, U, W) - w_lo + 1);
      float* slot = p.partial + (size_t)(gw - w_lo) * M * N;
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = (int)(rt * 16) + g + ((e & 2) ? 8 : 0);
          const int tok = j * 8 + 2 * t + (e & 1);
          if (row < N && tok < M) slot[(size_t)tok * N + row] = acc[j][e];
        }
      __threadfence();
      __syncwarp();
      int old = 0;
      if (lane == 0) old = atomicAdd(p.counters + rt, 1);
      old = __shfl_sync(0xffffffffu, old, 0);
      last = (old == n_contrib - 1);
      if (last) {
        if (lane == 0) p.counters[rt] = 0;
        __threadfence();
      }
    }
    if (!last) return;
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = (int)(rt * 16) + g + ((e & 2) ? 8 : 0);
        const int tok = j * 8 + 2 * t + (e & 1);
        if (row < N && tok < M) {
          float v = acc[j][e];
          if (!whole) {
            v = 0.f;
            for (int c = 0; c < n_contrib; ++c)
              v += __ldcg(p.partial + (size_t)c * M * N + (size_t)tok * N + row);
          }
          const size_t o = (size_t)tok * N + row;
          p.y[o] = epilogue(v, p.epi, p.operand, o);
        }
      }
  };

  for (long long base = u0; base < u1; base += P) {
#pragma unroll
    for (int i = 0; i < P; ++i) {
      const long long u = base + i;
      if (u >= u1) break;
      const Slot cur = ring[i];
      if (u + P < u1) load(u + P, ring[i]);

      const long long rt = u / B;
      const int kb = (int)(u - rt * B);
      float sa = cur.sa, sb = cur.sb;
      if (p.nested) {
        sa = nested_scale(code2_s[cur.qa], cur.sa, p.offset);
        sb = nested_scale(code2_s[cur.qb], cur.sb, p.offset);
      }
      float blk[NT][4];
#pragma unroll
      for (int j = 0; j < NT; ++j) blk[j][0] = blk[j][1] = blk[j][2] = blk[j][3] = 0.f;
      uint4 xr[NT][2];
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const int tok = j * 8 + g;
        if (tok < M) {
          const uint4* xp =
              reinterpret_cast<const uint4*>(p.x + (size_t)tok * K + (size_t)kb * 64 + t * 16);
          xr[j][0] = __ldg(xp);
          xr[j][1] = __ldg(xp + 1);
        } else {
          xr[j][0] = make_uint4(0, 0, 0, 0);
          xr[j][1] = make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const uint32_t wa = (s < 2) ? cur.wa.x : cur.wa.y;
        const uint32_t wb = (s < 2) ? cur.wb.x : cur.wb.y;
        const uint32_t sel0 = 0x5504u | ((uint32_t)(2 * (s & 1)) << 4);
        const uint32_t sel1 = 0x5504u | ((uint32_t)(2 * (s & 1) + 1) << 4);
        const uint32_t a0 = lut_lookup(lut, wa, sel0, lane_base);
        const uint32_t a2 = lut_lookup(lut, wa, sel1, lane_base);
        const uint32_t a1 = lut_lookup(lut, wb, sel0, lane_base);
        const uint32_t a3 = lut_lookup(lut, wb, sel1, lane_base);
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          const uint4& xs = xr[j][s >> 1];
          const uint32_t b0 = (s & 1) ? xs.z : xs.x;
          const uint32_t b1 = (s & 1) ? xs.w : xs.y;
          mma_bf16_16816(blk[j], a0, a1, a2, a3, b0, b1);
        }
      }
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        acc[j][0] = fmaf(sa, blk[j][0], acc[j][0]);
        acc[j][1] = fmaf(sa, blk[j][1], acc[j][1]);
        acc[j][2] = fmaf(sb, blk[j][2], acc[j][2]);
        acc[j][3] = fmaf(sb, blk[j][3], acc[j][3]);
      }
      if (kb == B - 1 || u == u1 - 1) {
        flush(rt);
#pragma unroll
        for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
      }
    }
  }
}

}  // namespace

static int g_sm_count[64];

int gemv_sm_count(int dev) {
  if (dev < 0 || dev >= 64) return 148;
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

void gemv_plan(int N, int K, int M, int sm_count, GemvPlan* plan) {
  const long long tiles = (N + 15) / 16;
  const long long B = K / 64;
  const long long U = tiles * B;
  const long long ctas = (long long)sm_count * GEMV_CTAS_PER_SM;
  long long W = ctas * kWarps;
  if (W > U) W = U;
  plan->tiles = tiles;
  plan->units = U;
  plan->warps_total = (int)W;
  plan->grid = (int)((W + kWarps - 1) / kWarps);
  // The longest run of warps that can share one tile: every warp owns at
  // least floor(U / W) units, so a tile of B units meets at most
  // ceil(B / floor(U / W)) + 1 of them.
  const long long per = U / W;
  plan->slots = (int)((B + per - 1) / per + 1);
  plan->counter_bytes = (size_t)((tiles * sizeof(int) + 255) / 256 * 256);
  plan->partial_bytes = (size_t)plan->slots * M * N * sizeof(float);
}

template <int NT>
static cudaError_t launch_nt(const GemvParams& p, int grid, cudaStream_t stream) {
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(nf4_gemv_kernel<NT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         GEMV_SMEM_BYTES);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = GEMV_SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, nf4_gemv_kernel<NT>, p);
}

cudaError_t launch_gemv(const GemvParams& p, int grid, cudaStream_t stream) {
  if (p.M <= 8) return launch_nt<1>(p, grid, stream);
  if (p.M <= 16) return launch_nt<2>(p, grid, stream);
  return launch_nt<4>(p, grid, stream);
}

}  // namespace nf4b
