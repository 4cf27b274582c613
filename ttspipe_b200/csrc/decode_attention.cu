// Grouped-query decode attention for one query position over a bf16 (or, F16,
// fp16) KV cache.
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
// Scores follow the fork's rounding: act(q.k) * head_dim^-0.5 in fp32, act the
// activation type.

#include "common.cuh"
#include "kernels.cuh"
#include "gemv_unit.cuh"
#include "tmap.cuh"

namespace nf4b {

namespace {

constexpr int kD = 128;
constexpr int kThreads = 128;

__device__ int g_attn_error = 0;  // bit 0: a bounded wait for the KV copies gave up

__device__ __forceinline__ uint32_t sm_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Bounded wait for phase 0 of `bar` (2 s by %globaltimer).
__device__ __forceinline__ bool wait_bar0(uint32_t bar) {
  unsigned long long start = 0;
  for (uint32_t i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar)
        : "memory");
    if (done) return true;
    if ((i & 63u) == 0u) {
      unsigned long long now;
      asm volatile("mov.u64 %0, %globaltimer;" : "=l"(now));
      if (i == 0) {
        start = now;
      } else if (now - start > 2000000000ull) {
        atomicOr(&g_attn_error, 1);
        return false;
      }
    }
  }
}

// Bounded wait for phase `parity` of `bar`.
__device__ __forceinline__ bool wait_bar_parity(uint32_t bar, uint32_t parity) {
  unsigned long long start = 0;
  for (uint32_t i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 63u) == 0u) {
      unsigned long long now;
      asm volatile("mov.u64 %0, %globaltimer;" : "=l"(now));
      if (i == 0) {
        start = now;
      } else if (now - start > 2000000000ull) {
        atomicOr(&g_attn_error, 1);
        return false;
      }
    }
  }
}

// Shared memory of one CTA: its chunk of K and V rows (copied whole by two
// bulk async copies), the group's queries, scores, partial-sum scratch.
template <int G>
struct AttnSmem {
  alignas(128) uint16_t k[ATTN_CHUNK * kD];
  alignas(128) uint16_t v[ATTN_CHUNK * kD];
  float q[G][kD];
  float sc[G][ATTN_CHUNK];
  float red[4][G][kD];
  float m[G], l[G];
  unsigned long long bar;
  int last;
};

template <int G, bool F16>
__global__ void __launch_bounds__(kThreads) decode_attention_kernel(
    const bf16_t* __restrict__ q, const bf16_t* __restrict__ kc, const bf16_t* __restrict__ vc,
    const int64_t* __restrict__ pos_ptr, const uint8_t* __restrict__ mask, bf16_t* __restrict__ out,
    int max_len, int window,
    int chunks, float scale, float* __restrict__ part_acc, float* __restrict__ part_ml,
    int* __restrict__ counters) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  AttnSmem<G>& sm = *reinterpret_cast<AttnSmem<G>*>(smem_raw);

  pdl_wait();  // the new K/V row and q come from the previous kernel
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
  const int rows = (int)(L - j0 < ATTN_CHUNK ? L - j0 : ATTN_CHUNK);
  const uint32_t bar = sm_u32(&sm.bar);
  if (tid == 0) {
    // rows j0 .. j0 + rows - 1 of this KV head are contiguous in both caches
    const uint32_t bytes = (uint32_t)rows * kD * 2;
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(2 * bytes) : "memory");
    const bf16_t* ksrc = kc + ((size_t)kh * max_len + j0) * kD;
    const bf16_t* vsrc = vc + ((size_t)kh * max_len + j0) * kD;
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     sm_u32(sm.k)),
                 "l"(ksrc), "r"(bytes), "r"(bar)
                 : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     sm_u32(sm.v)),
                 "l"(vsrc), "r"(bytes), "r"(bar)
                 : "memory");
  }
  for (int i = tid; i < G * kD; i += kThreads) sm.q[i / kD][i % kD] = act2f<F16>(q[(size_t)kh * G * kD + i]);
  __syncthreads();  // the barrier's initialisation is visible before anyone waits on it
  const bool ok = wait_bar0(bar);

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
      const bool vis = ok && (jl < rows) && (mask == nullptr || mask[j] != 0);
      if (vis) {
        const uint4* kr = reinterpret_cast<const uint4*>(sm.k + jl * kD + li * 16);
        const uint4 k0 = kr[0], k1 = kr[1];
        const uint32_t kw[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float ka = act_lo<F16>(kw[e]), kb = act_hi<F16>(kw[e]);
#pragma unroll
          for (int h = 0; h < G; ++h) {
            dot[h] = fmaf(sm.q[h][li * 16 + 2 * e], ka, dot[h]);
            dot[h] = fmaf(sm.q[h][li * 16 + 2 * e + 1], kb, dot[h]);
          }
        }
      }
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float v = dot[h];
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        if (li == 0) sm.sc[h][jl] = vis ? __fmul_rn(round_act<F16>(v), scale) : -INFINITY;
      }
    }
  }
  __syncthreads();

  // Chunk max and exp per head (a warp per head).
  for (int h = warp; h < G; h += 4) {
    const float a = sm.sc[h][lane], b = sm.sc[h][lane + 32];
    float m = fmaxf(a, b);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    const float pa = (a == -INFINITY) ? 0.f : expf(a - m);
    const float pb = (b == -INFINITY) ? 0.f : expf(b - m);
    sm.sc[h][lane] = pa;
    sm.sc[h][lane + 32] = pb;
    float l = pa + pb;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    if (lane == 0) {
      sm.m[h] = m;
      sm.l[h] = l;
    }
  }
  __syncthreads();

  // P.V: 16 dimension groups of 8 x 8 row groups of 8. Masked and past-the-end
  // rows are skipped, never multiplied by a zero weight.
  {
    const int dg = tid & 15, pg = tid >> 4;
    float acc[G][8];
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[h][e] = 0.f;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int jl = pg * 8 + r;
      if (!ok || jl >= rows) continue;
      if (mask != nullptr && mask[j0 + jl] == 0) continue;
      const uint4 vv = *reinterpret_cast<const uint4*>(sm.v + jl * kD + dg * 8);
      const uint32_t vw[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float p = sm.sc[h][jl];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          acc[h][2 * e] = fmaf(p, act_lo<F16>(vw[e]), acc[h][2 * e]);
          acc[h][2 * e + 1] = fmaf(p, act_hi<F16>(vw[e]), acc[h][2 * e + 1]);
        }
      }
    }
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float v = acc[h][e] + __shfl_xor_sync(0xffffffffu, acc[h][e], 16);
        if ((lane & 16) == 0) sm.red[warp][h][dg * 8 + e] = v;
      }
  }
  __syncthreads();
  for (int i = tid; i < G * kD; i += kThreads) {
    const int h = i / kD, d = i % kD;
    const float v = sm.red[0][h][d] + sm.red[1][h][d] + sm.red[2][h][d] + sm.red[3][h][d];
    const int qh = kh * G + h;
    part_acc[((size_t)qh * chunks + c) * kD + d] = v;
  }
  if (tid < G) {
    const int qh = kh * G + tid;
    part_ml[((size_t)qh * chunks + c) * 2] = sm.m[tid];
    part_ml[((size_t)qh * chunks + c) * 2 + 1] = sm.l[tid];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int old = atomicAdd(counters + kh, 1);
    sm.last = (old == active - 1);
    if (sm.last) counters[kh] = 0;
  }
  __syncthreads();
  if (!sm.last) {
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
    out[(size_t)qh * kD + d] = f2act<F16>(num / den);
  }
  pdl_launch_dependents();
}

// ---------------------------------------------------------------------------
// Cluster kernel: one thread-block cluster of C (= 8) CTAs per KV head. CTA r of the
// cluster takes a contiguous share of the live rows, streams it through a
// two-stage ring of 64-row K/V chunks (two bulk async copies per chunk, both
// contiguous in the cache) with an fp32 online softmax, and leaves its
// unnormalised partial (max, sum, output) in its shared memory. After a
// cluster barrier, CTA 0 merges the C partials in rank order through
// distributed shared memory and writes the output: one launch, no global
// partials, no atomics.
// ---------------------------------------------------------------------------

// 8 warps. (16 warps for groups of <= 4 query heads measured 0.6 us faster
// at 2048 rows, four chunks per CTA, but 0.8-1 us slower for windows of one
// or two chunks per CTA, which the fast AR and most slow-AR positions use.)
// Warp w takes key rows 8w .. 8w + 7 of every 64-row chunk.
template <int G>
__host__ __device__ constexpr int cthreads() { return 256; }
static_assert(ATTN_CHUNK == 8 * (256 / 32), "a chunk is 8 key rows per warp");

// Stages of the cluster kernel's K/V ring: every chunk of a CTA's share is in
// flight at once up to this depth (a 2048-row window over 8 CTAs is 4 chunks
// each), so the chunks' copy latencies overlap instead of adding up.
constexpr int kCStages = 4;

template <int G>
struct ClusterSmem {
  // [stage][K, V]: 64 rows x 128 dims as two 8 KB boxes (dims 0-63, 64-127),
  // each written by a 2-D TMA copy in the 128-byte swizzle: row r's 16-byte
  // chunk c sits at chunk c ^ (r & 7) of its 128-byte line (kv_off).
  alignas(1024) uint16_t kv[kCStages][2][ATTN_CHUNK * kD];
  float q[G][kD];
  float red[cthreads<G>() / 32][G][kD];  // each warp's partial output
  float wm[cthreads<G>() / 32][G], wl[cthreads<G>() / 32][G];  // and its max and sum
  float part_acc[G][kD];
  float part_m[G], part_l[G];
  // the cluster merge's inbox: slot r holds what rank r pushed (its output
  // partial for this CTA's share of the outputs, its max and sum per head)
  float in_acc[8][G * kD];
  float in_m[8][G], in_l[8][G];
  unsigned long long bar[kCStages];
  // the fused q/k norm + rotary prologue (QkvIn)
  float sx[2][kD];
  double nred[cthreads<G>() / 32];
  uint16_t knew[kD], vnew[kD];
};

// Byte offset of (row r, dimension d) in a K or V stage (see ClusterSmem::kv).
__device__ __forceinline__ uint32_t kv_off(int r, int d) {
  return (uint32_t)((d >> 6) * 8192 + r * 128 + ((((d >> 3) & 7) ^ (r & 7)) << 4) + ((d & 7) << 1));
}

// One 64-dimension x 64-row box of a K or V cache (a 2-D map over
// [n_kv * max_len rows, 128 dims]; rows past the end are zero-filled).
__device__ __forceinline__ void tma_box(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Four 8x8 16-bit matrices, transposed (MMA B fragments of a [k][n] row-major tile).
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Store v at the address `local` names in the shared memory of cluster rank `rank`.
__device__ __forceinline__ void st_cluster_f32(float* local, uint32_t rank, float v) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(sm_u32(local)), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

// One 128-wide row per half of the first 256 threads (threads 0-127: half 0,
// 128-255: half 1; the others only join the barriers)
// with qk_rope_kv's arithmetic: RMSNorm with this half's weight w (none when
// null) - fp64 sum of squares, reduced exactly as block_sum over 4 warps -
// then the rotary pair (x0 c - x1 s, x1 c + x0 s) at the freqs row when
// `rope`. Every thread calls it (uniform barriers); `any_norm` is uniform.
template <int G, bool F16>
__device__ __forceinline__ float norm_rope_half(ClusterSmem<G>& sm, float x, bool has_w, float wd, bool rope,
                                                bool any_norm, float eps, float c, float sn) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int d = tid & (kD - 1), half = (tid >> 7) & 1;
  const bool mine = tid < 2 * kD;
  if (any_norm) {
    double sq = has_w ? (double)x * (double)x : 0.0;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
    if (lane == 0) sm.nred[warp] = sq;
    __syncthreads();
    double ss = 0.0;
#pragma unroll
    for (int i = 0; i < 4; ++i) ss += sm.nred[4 * half + i];
    if (has_w) {
      const float r = rsqrt_exact(ss, kD, eps);
      x = round_act<F16>(__fmul_rn(__fmul_rn(x, r), wd));
    }
    __syncthreads();
  }
  if (mine) sm.sx[half][d] = x;
  __syncthreads();
  float y = x;
  if (rope) {
    const float x0 = sm.sx[half][d & ~1], x1 = sm.sx[half][d | 1];
    y = (d & 1) ? __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, sn)) : __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
  }
  __syncthreads();
  return y;
}

template <int G, bool F16>
__global__ void __launch_bounds__(cthreads<G>()) decode_attention_cluster_kernel(
    const bf16_t* __restrict__ q, const bf16_t* __restrict__ kc, const bf16_t* __restrict__ vc,
    const int64_t* __restrict__ pos_ptr, const uint8_t* __restrict__ mask, bf16_t* __restrict__ out,
    int max_len, int window, float scale, const QkvIn in, const __grid_constant__ CUtensorMap tmk,
    const __grid_constant__ CUtensorMap tmv) {
  constexpr int kCT = cthreads<G>();
  extern __shared__ __align__(128) uint8_t smem_raw[];
  // 1024-byte aligned for the swizzled boxes (the launch adds 1 KB of slack);
  // the same offset in every CTA of a cluster, as the merge's mapa needs
  ClusterSmem<G>& sm = *reinterpret_cast<ClusterSmem<G>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                          ~(uintptr_t)1023);
  const int kh = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t rank = cluster_rank(), C = cluster_size();
  // A CTA may store into another CTA's shared memory only once every CTA of
  // the cluster is running: every thread arrives here and waits just before
  // the merge's first push, by when the others have long arrived.
  if (C > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");

  pdl_wait();  // the new K/V row and q come from the previous kernel
  // The next kernel (the wo GEMV) may be scheduled now: its CTAs load their
  // first weights on the SMs this grid leaves free; it reads this kernel's
  // output only after its own dependency wait, which waits for this grid to
  // complete.
  pdl_launch_dependents();
  // A window of one chunk read by one CTA (the fast AR's): its rows' copies go
  // out before the position is read - the whole window, rows past the live
  // length are never used - saving a round trip.
  const bool whole_window = C == 1 && window <= ATTN_CHUNK;
  // Every chunk is four whole boxes (K and V, two 64-dimension halves each),
  // 32 KB of transaction bytes whatever its live rows.
  auto copy_chunk = [&](int stg, long long row0) {  // one thread
    const uint32_t bar = sm_u32(&sm.bar[stg]);
    const int y = (int)((long long)kh * max_len + row0);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(4 * 8192) : "memory");
    tma_box(sm_u32(sm.kv[stg][0]), &tmk, 0, y, bar);
    tma_box(sm_u32(sm.kv[stg][0]) + 8192, &tmk, 64, y, bar);
    tma_box(sm_u32(sm.kv[stg][1]), &tmv, 0, y, bar);
    tma_box(sm_u32(sm.kv[stg][1]) + 8192, &tmv, 64, y, bar);
  };
  if (whole_window && threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sm_u32(&sm.bar[0])) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sm_u32(&sm.bar[1])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    copy_chunk(0, 0);
  }
  long long L = (pos_ptr != nullptr) ? pos_ptr[0] + 1 : (long long)window;
  if (L > window) L = window;
  if (L < 1) L = 1;
  // This CTA's rows: a contiguous share, whole 64-row chunks except at the end.
  const long long nch = (L + ATTN_CHUNK - 1) / ATTN_CHUNK;
  const long long per = (nch + C - 1) / C;
  const long long r0 = (long long)rank * per * ATTN_CHUNK;
  long long r1 = r0 + per * ATTN_CHUNK;
  if (r1 > L) r1 = L;
  const int my_chunks = r1 > r0 ? (int)((r1 - r0 + ATTN_CHUNK - 1) / ATTN_CHUNK) : 0;
  // thread 0: chunk ci into stage ci % kCStages
  auto issue = [&](int ci) { copy_chunk(ci % kCStages, r0 + (long long)ci * ATTN_CHUNK); };
  if (tid == 0 && !whole_window) {
    for (int i = 0; i < kCStages; ++i)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sm_u32(&sm.bar[i])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int ci = 0; ci < kCStages && ci < my_chunks; ++ci) issue(ci);
  }
  const bool fused = in.qkv != nullptr;  // q/k/v from the wqkv output (pos given, no mask)
  const long long p_new = fused ? pos_ptr[0] : -1;
  if (!fused) {
    // every load first (one round trip), then the stores
    constexpr int QN = (G * kD + kCT - 1) / kCT;
    uint16_t qv[QN];
#pragma unroll
    for (int j = 0; j < QN; ++j) {
      const int i = tid + j * kCT;
      qv[j] = i < G * kD ? __ldg(q + (size_t)kh * G * kD + i) : (uint16_t)0;
    }
#pragma unroll
    for (int j = 0; j < QN; ++j) {
      const int i = tid + j * kCT;
      if (i < G * kD) sm.q[i / kD][i % kD] = act2f<F16>(qv[j]);
    }
  } else {
    // This KV head's query heads, two per pass, then k (half 0) and v (half 1):
    // the arithmetic of qk_rope_kv. The new rows reach the cache through rank 0;
    // the CTA whose chunk holds row p_new patches them into its shared copy.
    const int d = tid & (kD - 1), half = (tid >> 7) & 1;
    const bool mine = tid < 2 * kD;  // threads 256+ only join the barriers
    const bf16_t* qkv = in.qkv;
    const bool norm = in.qw != nullptr;  // q and k norm weights come together
    // every global load first (one round trip), then the passes
    constexpr int P = (G + 1) / 2;
    float xq[P];
#pragma unroll
    for (int i = 0; i < P; ++i) {
      const int h = 2 * i + half;
      xq[i] = h < G ? act2f<F16>(qkv[(size_t)(kh * G + h) * kD + d]) : 0.f;
    }
    const int nkv = (int)gridDim.x;
    const float xkv = act2f<F16>(qkv[(size_t)(in.n_head + (half ? nkv : 0) + kh) * kD + d]);
    const float c = load_freq(in.freqs, d & ~1, in.ftype), sn = load_freq(in.freqs, d | 1, in.ftype);
    const float qwd = norm ? act2f<F16>(in.qw[d]) : 0.f, kwd = norm ? act2f<F16>(in.kw[d]) : 0.f;
#pragma unroll
    for (int i = 0; i < P; ++i) {
      const int h = 2 * i + half;
      const float y = norm_rope_half<G, F16>(sm, xq[i], norm, qwd, true, norm, in.eps, c, sn);
      if (h < G && mine) sm.q[h][d] = round_act<F16>(y);
    }
    const float y = norm_rope_half<G, F16>(sm, xkv, norm && half == 0, kwd, half == 0, norm, in.eps, c, sn);
    const bf16_t nb = f2act<F16>(y);
    if (mine) (half ? sm.vnew : sm.knew)[d] = nb;
    if (mine && rank == 0 && p_new < max_len) {
      bf16_t* cache = const_cast<bf16_t*>(half ? vc : kc);
      cache[((size_t)kh * max_len + p_new) * kD + d] = nb;
    }
  }
  __syncthreads();

  // Tensor-core form (mma.sync m16n8k16, fp32 accumulators): the query heads
  // are the A rows (G of 16 used), warp w's 8 key rows of a chunk the score
  // tile's columns, so lane (g, t) = (lane / 4, lane % 4) gets head g's
  // scores for keys 8w + 2t and 8w + 2t + 1, and those two values, rounded to
  // the activation type, are already its A fragment for the P.V product
  // (keys as k, the 128 dimensions as 16 column tiles). Each warp keeps its own
  // online softmax (max, sum, output) for its rows; the eight are merged once
  // at the end.
  const int g = lane >> 2, t = lane & 3;
  uint32_t qa[8][2];  // A fragments of the 8 k steps: dims 16s + 2t (+1) and 16s + 2t + 8 (+9)
#pragma unroll
  for (int st = 0; st < 8; ++st) {
    const int d0 = 16 * st + 2 * t;
    qa[st][0] = g < G ? pack_act2<F16>(sm.q[g < G ? g : 0][d0], sm.q[g < G ? g : 0][d0 + 1]) : 0u;
    qa[st][1] = g < G ? pack_act2<F16>(sm.q[g < G ? g : 0][d0 + 8], sm.q[g < G ? g : 0][d0 + 9]) : 0u;
  }
  float acc[16][4];  // output tile j: head g, dimensions 8j + 2t, 8j + 2t + 1 (and unused head g + 8)
#pragma unroll
  for (int j = 0; j < 16; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  float wmax = -INFINITY, wsum = 0.f;  // this warp's running max and sum for head g
  const int kr = 8 * warp + g;         // the key row of this lane's score B fragments
  const int vr = 8 * warp + (lane & 7);  // the key row whose address this lane gives ldmatrix
  bool ok = true;
  for (int ci = 0; ci < my_chunks; ++ci) {
    const int stg = ci % kCStages;
    // one decision for the whole CTA: a chunk whose copy never lands stops it
    if (!__syncthreads_and(wait_bar_parity(sm_u32(&sm.bar[stg]), (uint32_t)(ci / kCStages) & 1u))) {
      ok = false;
      if (tid == 0) {
        // the copies still in flight (chunks ci .. the last issued) land before the
        // CTA releases its shared memory - within one more bounded wait each
        for (int cj = ci; cj < my_chunks && cj < ci + kCStages; ++cj)
          if (!wait_bar_parity(sm_u32(&sm.bar[cj % kCStages]), (uint32_t)(cj / kCStages) & 1u)) break;
      }
      __syncthreads();
      break;
    }
    const long long j0 = r0 + (long long)ci * ATTN_CHUNK;
    const int rows = (int)((r1 - j0 < ATTN_CHUNK) ? r1 - j0 : ATTN_CHUNK);
    uint8_t* kst = reinterpret_cast<uint8_t*>(sm.kv[stg][0]);
    uint8_t* vst = reinterpret_cast<uint8_t*>(sm.kv[stg][1]);
    if (fused && p_new >= j0 && p_new < j0 + rows) {
      // the copy may predate rank 0's store of the new row: use the computed one
      const int d = tid & (kD - 1), half = tid >> 7;
      if (half < 2)
        *reinterpret_cast<uint16_t*>((half ? vst : kst) + kv_off((int)(p_new - j0), d)) =
            (half ? sm.vnew : sm.knew)[d];
      __syncthreads();
    }
    // Rows that are masked or past the live length: their V rows are zeroed
    // before the P.V product (their weights are zero, and whatever the stage
    // holds - NaN included - must not reach the sums); their scores are
    // replaced by -inf below, whatever the K bytes hold.
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int jl = 8 * warp + i;
      const bool live = jl < rows && (mask == nullptr || mask[j0 + jl] != 0);
      if (!live && lane < 16) *reinterpret_cast<uint4*>(vst + (lane >> 3) * 8192 + jl * 128 + (lane & 7) * 16) =
          make_uint4(0u, 0u, 0u, 0u);
    }
    __syncwarp();
    // Scores: 8 k steps of 16 dimensions; the B fragment words of key row kr
    // (dims 16s + 2t, +1 and 16s + 2t + 8, +9) are conflict-free thanks to the swizzle.
    float sd[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int st = 0; st < 8; ++st) {
      const int d0 = 16 * st + 2 * t;
      const uint32_t b0 = *reinterpret_cast<const uint32_t*>(kst + kv_off(kr, d0));
      const uint32_t b1 = *reinterpret_cast<const uint32_t*>(kst + kv_off(kr, d0 + 8));
      mma_act<F16>(sd, qa[st][0], 0u, qa[st][1], 0u, b0, b1);
    }
    const int k0 = 8 * warp + 2 * t;
    const bool vis0 = k0 < rows && (mask == nullptr || mask[j0 + k0] != 0);
    const bool vis1 = k0 + 1 < rows && (mask == nullptr || mask[j0 + k0 + 1] != 0);
    const float s0 = vis0 ? __fmul_rn(round_act<F16>(sd[0]), scale) : -INFINITY;
    const float s1 = vis1 ? __fmul_rn(round_act<F16>(sd[1]), scale) : -INFINITY;
    // Online softmax of head g over this warp's rows (the quad t = 0..3).
    float mc = fmaxf(s0, s1);
    mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, 1));
    mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, 2));
    const float mn = fmaxf(wmax, mc);
    const float al = (mn == -INFINITY) ? 1.f : expf(wmax - mn);
    const float p0 = (s0 == -INFINITY) ? 0.f : expf(s0 - mn);
    const float p1 = (s1 == -INFINITY) ? 0.f : expf(s1 - mn);
    const uint32_t pa = pack_act2<F16>(p0, p1);  // the weights as the P.V product uses them
    float ls = act_lo<F16>(pa) + act_hi<F16>(pa);
    ls += __shfl_xor_sync(0xffffffffu, ls, 1);
    ls += __shfl_xor_sync(0xffffffffu, ls, 2);
    wsum = wsum * al + ls;
    wmax = mn;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      acc[j][0] *= al;
      acc[j][1] *= al;
    }
    // P.V: four transposed ldmatrix loads (32 dimensions each) give the B
    // fragments of the 16 column tiles; keys 8..15 of the k step are absent
    // (zero A and B halves).
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) {
      uint32_t b[4];
      ldsm_x4_trans(b, sm_u32(vst) + kv_off(vr, 32 * q4 + 8 * (lane >> 3)));
#pragma unroll
      for (int m = 0; m < 4; ++m) mma_act<F16>(acc[4 * q4 + m], pa, 0u, 0u, 0u, b[m], 0u);
    }
    __syncthreads();  // every thread is done with this stage
    if (tid == 0 && ci + kCStages < my_chunks) issue(ci + kCStages);
  }
  // This CTA's partial: the eight warps' partials merged in warp order.
  if (g < G) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      sm.red[warp][g][8 * j + 2 * t] = acc[j][0];
      sm.red[warp][g][8 * j + 2 * t + 1] = acc[j][1];
    }
    if (t == 0) {
      sm.wm[warp][g] = wmax;
      sm.wl[warp][g] = wsum;
    }
  }
  __syncthreads();
  if (C > 1) asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // every CTA is running
  for (int i = tid; i < G * kD; i += kCT) {
    const int h = i / kD, d = i % kD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kCT / 32; ++w) M = fmaxf(M, sm.wm[w][h]);
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int w = 0; w < kCT / 32; ++w) {
      const float e = (sm.wm[w][h] == -INFINITY) ? 0.f : expf(sm.wm[w][h] - M);
      num = fmaf(sm.red[w][h][d], e, num);
      den = fmaf(sm.wl[w][h], e, den);
    }
    sm.part_acc[h][d] = num;
    if (d == 0) {
      sm.part_m[h] = M;
      sm.part_l[h] = den;
    }
    if (C > 1) {
      // push this partial to the rank that merges output i, and the head's
      // max and sum to every rank (they arrive before the cluster barrier)
      // the owner of i: the largest q with floor(q E / C) <= i (the merge's shares)
      st_cluster_f32(&sm.in_acc[rank][i], (uint32_t)(((long long)(i + 1) * C - 1) / (G * kD)), num);
      if (d == 0)
        for (uint32_t q = 0; q < C; ++q) {
          st_cluster_f32(&sm.in_m[rank][h], q, M);
          st_cluster_f32(&sm.in_l[rank][h], q, den);
        }
    }
  }
  if (C == 1) {
    // One CTA per KV head: its partial is the result (the merge below with a
    // single partial has weight exp(0) = 1, so this is bit for bit the same).
    __syncthreads();
    for (int i = tid; i < G * kD; i += kCT) {
      const int h = i / kD, d = i % kD;
      const float w = (sm.part_m[h] == -INFINITY) ? 0.f : 1.f;
      out[(size_t)(kh * G + h) * kD + d] = f2act<F16>(fmaf(sm.part_acc[h][d], w, 0.f) / fmaf(sm.part_l[h], w, 0.f));
    }
    return;
  }
  // Every rank's pushes land before the barrier completes (release / acquire);
  // after it each CTA reads only its own shared memory, so no CTA waits for
  // another to finish reading before it may exit.
  cluster_sync();
  {
    // Each CTA of the cluster merges its share of the (head, dimension)
    // outputs from the partials the ranks pushed, in rank order.
    const int E = G * kD, lo = (int)(rank * E / C), hi = (int)((rank + 1) * E / C);
    for (int i = lo + tid; i < hi; i += kCT) {
      const int h = i / kD, d = i % kD;
      float M = -INFINITY;
      for (uint32_t r = 0; r < C; ++r) M = fmaxf(M, sm.in_m[r][h]);
      float num = 0.f, den = 0.f;
      for (uint32_t r = 0; r < C; ++r) {
        const float m = sm.in_m[r][h];
        const float w = (m == -INFINITY) ? 0.f : expf(m - M);
        den = fmaf(sm.in_l[r][h], w, den);
        num = fmaf(sm.in_acc[r][i], w, num);
      }
      out[(size_t)(kh * G + h) * kD + d] = f2act<F16>(num / den);
    }
  }
}

}  // namespace

int read_attn_error(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_attn_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_attn_error, &zero, sizeof(int));
  }
  return v;
}

void attn_plan(int n_head, int head_dim, int window, AttnPlan* plan) {
  plan->chunks = (window + ATTN_CHUNK - 1) / ATTN_CHUNK;
  plan->counter_bytes = ATTN_COUNTER_BYTES;
  plan->partial_bytes = (size_t)n_head * plan->chunks * (head_dim + 2) * sizeof(float);
}

namespace {

template <int G, bool F16>
cudaError_t launch_cluster_g(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int64_t* pos,
                             const uint8_t* mask, uint16_t* out, int nkv, int max_len, int window, int C,
                             bool check, const QkvIn& in, cudaStream_t stream) {
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int smem = (int)sizeof(ClusterSmem<G>) + 1024;  // + slack for the 1024-byte alignment
  // K and V caches as 2-D [n_kv * max_len rows, 128 dims] maps, 64 x 64 boxes
  // in the 128-byte swizzle (base and row stride are 16-byte multiples).
  CUtensorMap mk, mv;
  const uint64_t rows = (uint64_t)nkv * (uint64_t)max_len;
  if (!make_map_2d(&mk, CU_TENSOR_MAP_DATA_TYPE_UINT16, kc, kD, rows, kD * 2, 64, ATTN_CHUNK,
                   CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_2d(&mv, CU_TENSOR_MAP_DATA_TYPE_UINT16, vc, kD, rows, kD * 2, 64, ATTN_CHUNK,
                   CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(decode_attention_cluster_kernel<G, F16>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nkv, C);
  cfg.blockDim = dim3(cthreads<G>());
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  // One CTA per KV head (a one-chunk window) needs no cluster: a plain launch
  // is an implicit cluster of one for the kernel's cluster operations.
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = C;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = C > 1 ? 2 : 1;
  int clusters = 1;
  if (check && C > 1 &&
      (cudaOccupancyMaxActiveClusters(&clusters, decode_attention_cluster_kernel<G, F16>, &cfg) != cudaSuccess ||
       clusters < 1)) {
    (void)cudaGetLastError();
    return cudaErrorNotSupported;
  }
  const float scale = 1.0f / sqrtf((float)kD);
  return cudaLaunchKernelEx(&cfg, decode_attention_cluster_kernel<G, F16>, (const bf16_t*)q, (const bf16_t*)kc,
                            (const bf16_t*)vc, pos, mask, (bf16_t*)out, max_len, window, scale, in, mk, mv);
}

}  // namespace

cudaError_t launch_cluster_attention(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int64_t* pos,
                                     const uint8_t* mask, uint16_t* out, int nh, int nkv, int max_len, int window,
                                     cudaStream_t stream, const QkvIn& in, bool f16) {
  // Clusters of 8 (the portable size; 16 measured slower at every window
  // length, 18.6 against 9.3 us at 512 rows, 24.4 against 17.1 at 2048);
  // fewer when the window has fewer 64-row chunks (a window of one chunk -
  // the fast AR's - runs one CTA per KV head, no cross-CTA merge). chosen:
  // 0 unknown, 1 launches, -1 cannot be resident.
  static int chosen[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int groups = nh / nkv;
  const int idx = (dev >= 0 && dev < 64) ? dev : 0;
  if (chosen[idx] < 0) return cudaErrorNotSupported;
  {
    const int chunks = (window + ATTN_CHUNK - 1) / ATTN_CHUNK;
    const int C = chunks < 8 ? (chunks < 1 ? 1 : chunks) : 8;
    const bool check = chosen[idx] == 0;
    cudaError_t e;
    switch (groups) {
      case 1:
        e = f16 ? launch_cluster_g<1, true>(q, kc, vc, pos, mask, out, nkv, max_len, window, C, check, in, stream)
                : launch_cluster_g<1, false>(q, kc, vc, pos, mask, out, nkv, max_len, window, C, check, in, stream);
        break;
      case 2:
        e = f16 ? launch_cluster_g<2, true>(q, kc, vc, pos, mask, out, nkv, max_len, window, C, check, in, stream)
                : launch_cluster_g<2, false>(q, kc, vc, pos, mask, out, nkv, max_len, window, C, check, in, stream);
        break;
      case 4:
        e = f16 ? launch_cluster_g<4, true>(q, kc, vc, pos, mask, out, nkv, max_len, window, C, check, in, stream)
                : launch_cluster_g<4, false>(q, kc, vc, pos, mask, out, nkv, max_len, window, C, check, in, stream);
        break;
      case 8:
        e = f16 ? launch_cluster_g<8, true>(q, kc, vc, pos, mask, out, nkv, max_len, window, C, check, in, stream)
                : launch_cluster_g<8, false>(q, kc, vc, pos, mask, out, nkv, max_len, window, C, check, in, stream);
        break;
      default: return cudaErrorInvalidValue;
    }
    if (e == cudaSuccess) {
      chosen[idx] = 1;
      return e;
    }
    (void)cudaGetLastError();
    // Only a cluster that cannot be resident is a property of the device; a
    // call whose caches the tensor maps reject (an argument of this call) falls
    // back for this call alone.
    if (e != cudaErrorNotSupported) return e;
  }
  chosen[idx] = -1;
  return cudaErrorNotSupported;
}

cudaError_t launch_decode_attention(const uint16_t* q, const uint16_t* kc, const uint16_t* vc,
                                    const int64_t* pos, const uint8_t* mask, uint16_t* out, int nh, int nkv,
                                    int max_len, int window, float* partial, int* counters,
                                    cudaStream_t stream, bool f16) {
  const int groups = nh / nkv;
  const int chunks = (window + ATTN_CHUNK - 1) / ATTN_CHUNK;
  {
    // One cluster of 8 CTAs per KV head; the split-KV kernel below if the
    // device cannot make such a cluster resident.
    const QkvIn none = {};
    cudaError_t e = launch_cluster_attention(q, kc, vc, pos, mask, out, nh, nkv, max_len, window, stream, none, f16);
    if (e == cudaSuccess) return e;
    (void)cudaGetLastError();
  }
  float* part_acc = partial;
  float* part_ml = partial + (size_t)nh * chunks * kD;
  const float scale = 1.0f / sqrtf((float)kD);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nkv, chunks);
  cfg.blockDim = dim3(kThreads);
  cfg.stream = stream;
  static bool configured[2][4][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int gi = groups == 1 ? 0 : groups == 2 ? 1 : groups == 4 ? 2 : 3;
  auto launch = [&](auto kernel, size_t smem) -> cudaError_t {
    cfg.dynamicSmemBytes = smem;
    if (dev >= 0 && dev < 64 && !configured[f16][gi][dev]) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      configured[f16][gi][dev] = true;
    }
    return cudaLaunchKernelEx(&cfg, kernel, (const bf16_t*)q, (const bf16_t*)kc, (const bf16_t*)vc, pos, mask,
                              (bf16_t*)out, max_len, window, chunks, scale, part_acc, part_ml, counters);
  };
#define NF4B_ATTN_CASE(GG)                                                                       \
  case GG:                                                                                       \
    return f16 ? launch(decode_attention_kernel<GG, true>, sizeof(AttnSmem<GG>))                  \
               : launch(decode_attention_kernel<GG, false>, sizeof(AttnSmem<GG>));
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

cudaError_t launch_qkv_attention(const QkvIn& in, const int64_t* pos, uint16_t* q_scratch, uint16_t* kc,
                                 uint16_t* vc, uint16_t* out, int nh, int nkv, int max_len, int window,
                                 float* partial, int* counters, cudaStream_t stream, bool f16) {
  cudaError_t e =
      launch_cluster_attention(nullptr, kc, vc, pos, nullptr, out, nh, nkv, max_len, window, stream, in, f16);
  if (e == cudaSuccess) return e;
  (void)cudaGetLastError();
  e = launch_qk_rope_kv(in.qkv, in.qw, in.kw, in.eps, in.freqs, in.ftype, pos, q_scratch, kc, vc, nh, nkv, max_len,
                        stream, f16);
  if (e != cudaSuccess) return e;
  return launch_decode_attention(q_scratch, kc, vc, pos, nullptr, out, nh, nkv, max_len, window, partial, counters,
                                 stream, f16);
}

}  // namespace nf4b
