// Streaming NF4 GEMV for decode (1..32 activation rows) on sm_100a.
//
// Replaces the reference's `nf4_mma` kernel for N <= 32 inputs
// (app/engine/nf4gemv.py:108-231, launch configs :234-248).
//
// Work decomposition. A "unit" is 16 weight rows x a k span (128 codes for
// the pair kernel, 64 for the block kernel). Units are numbered row-tile-major
// and split into equal contiguous runs, one run per warp of a persistent grid
// sized to the SM count, so every SM streams the same number of bytes whatever
// the weight shape. A warp that owns a whole row tile stores its outputs
// directly; tiles split between warps are reduced through a workspace: each
// contributor writes its fp32 partial into its own slot, and the last to
// arrive (an atomic counter per tile) sums the slots in slot order -
// deterministic - applies the epilogue and re-zeroes the counter. No warp ever
// waits on another.
//
// Inner loop. Each lane loads packed bytes of two rows (g and g+8), turns every
// byte into a bf16x2 pair of NF4 code values with ONE shared-memory load (a
// 256-entry pair table with one copy per lane, so the 32 lanes always hit 32
// different banks; the address is built with a single byte-permute), and
// feeds the pairs as the A fragment of mma.m16n8k16 with x as B. The scale
// of each 64-block multiplies that block's fp32 partial afterwards:
// y = sum_b s_b * sum_k code[q_k] x_k, the factorisation of the reference's
// CPU kernel (app/engine/nf4cpu.py:104-131).
//
//  * pair kernel (rows <= 4, k_in % 128 == 0): a lane loads 16 bytes of each of
//    its two rows (two 64-blocks per 4-lane group); the MMA's 8 columns carry
//    (activation row, block parity), so one MMA sums both blocks into separate
//    columns and each block still gets its own scale.
//  * block kernel (rows <= 32): a lane loads 8 bytes per row (the group covers
//    one 64-block); columns are activation rows, up to 4 column tiles.
//
// Weights are read with 256-byte L2 prefetch and no L1 allocation, several
// units ahead; x through L1. Programmatic dependent launch: the tables and
// the first weight loads are issued before `griddepcontrol.wait`, overlapping
// the previous kernel's tail; x, the workspace and y are touched only after it.

#include <type_traits>

#include "common.cuh"
#include "kernels.cuh"
#include "tmap.cuh"
#include "gemv_unit.cuh"

#ifndef NF4B_GEMV_PREFETCH_EARLY
#define NF4B_GEMV_PREFETCH_EARLY 1  // stream the hinted weight into L2 at kernel start (0: at the end)
#endif

namespace nf4b {

namespace {

constexpr int kWarps = GEMV_WARPS;
constexpr int kThreads = kWarps * 32;

// The warp whose unit run contains unit u (runs of uq + 1 units for the first
// ur warps, uq after them).
__device__ __forceinline__ int warp_of(int u, int uq, int ur) {
  const int big = ur * (uq + 1);
  return u < big ? u / (uq + 1) : ur + (u - big) / uq;
}

__device__ __forceinline__ int atomic_add_acq_rel(int* addr, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(addr), "r"(v) : "memory");
  return old;
}

// Shared-memory tables: the NF4 pair table and (nested scales) code2. Entry
// e's 32 per-lane copies are 128 contiguous bytes (stride 256), written eight
// copies per 16-byte store.
// The pair table alone (entry e's 32 per-lane copies at e * 256).
template <int THREADS>
__device__ __forceinline__ void build_pair_lut(uint8_t* smem) {
  for (int i = threadIdx.x; i < 256 * 8; i += THREADS) {
    const int e = i >> 3, part = i & 7;
    const uint32_t v = pack_bf16x2(nf4_code_imm((uint32_t)e >> 4), nf4_code_imm((uint32_t)e & 15u));
    *reinterpret_cast<uint4*>(smem + e * 256 + part * 16) = make_uint4(v, v, v, v);
  }
}

template <int THREADS = kThreads>
__device__ __forceinline__ void build_tables(uint8_t* smem, const GemvParams& p) {
  for (int i = threadIdx.x; i < 256 * 8; i += THREADS) {
    const int e = i >> 3, part = i & 7;
    const uint32_t v = pack_bf16x2(nf4_code_imm((uint32_t)e >> 4), nf4_code_imm((uint32_t)e & 15u));
    *reinterpret_cast<uint4*>(smem + e * 256 + part * 16) = make_uint4(v, v, v, v);
  }
  if (p.nested) {
    float* code2_s = reinterpret_cast<float*>(smem + GEMV_LUT_BYTES);
    for (int i = threadIdx.x; i < 256; i += THREADS) code2_s[i] = p.code2[i];
    if (p.code2_3 != nullptr)
      for (int i = threadIdx.x; i < 256; i += THREADS) code2_s[256 + i] = p.code2_3[i];
  }
}

// Finish row tile `rt`: every lane holds NV (row, activation row, value)
// triples. A warp that covered the whole tile stores directly; otherwise the
// split-tile protocol described at the top of this file.
template <int NV>
__device__ __forceinline__ void finish_tile(const GemvParams& p, int rt, int u0, int u1, int gw,
                                            const int (&row)[NV], const int (&tok)[NV],
                                            const float (&val)[NV], int lane) {
  const int t0 = rt * p.blocks_per_tile, t1 = t0 + p.blocks_per_tile - 1;
  const bool whole = (t0 >= u0) && (t1 < u1);
  const int N = p.N, M = p.M;
  int n_contrib = 1;
  if (!whole) {
    const int w_lo = warp_of(t0, p.uq, p.ur);
    n_contrib = warp_of(t1, p.uq, p.ur) - w_lo + 1;
    float* slot = p.partial + (size_t)(gw - w_lo) * M * N;
#pragma unroll
    for (int e = 0; e < NV; ++e)
      if (row[e] < N && tok[e] < M) slot[(size_t)tok[e] * N + row[e]] = val[e];
    // The warp barrier orders every lane's partial before lane 0's release
    // (fence + arrival); the last arriver's acquire orders the reads after it.
    __syncwarp();
    int old = 0;
    if (lane == 0) {
      asm volatile("fence.acq_rel.gpu;" ::: "memory");
      old = atomic_add_acq_rel(p.counters + rt, 1);
    }
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old != n_contrib - 1) return;
    if (lane == 0) p.counters[rt] = 0;
    __syncwarp();
  }
#pragma unroll
  for (int e = 0; e < NV; ++e) {
    if (row[e] < N && tok[e] < M) {
      float v = val[e];
      if (!whole) {
        v = 0.f;
        for (int c = 0; c < n_contrib; ++c)
          v += __ldcg(p.partial + (size_t)c * M * N + (size_t)tok[e] * N + row[e]);
      }
      const size_t o = (size_t)tok[e] * N + row[e];
      p.y[o] = epilogue(v, p.epi, p.operand, o);
    }
  }
}

// This warp's share of the hinted ranges, streamed into L2.
__device__ __forceinline__ void prefetch_next(const GemvParams& p, int gw, int lane) {
  if (lane == 0) prefetch_share(p.pf, gw, p.warps_total);
}

// ---------------------------------------------------------------------------
// pair kernel: units of 16 rows x 128 codes, activation rows <= 4
// ---------------------------------------------------------------------------

// Sums of the `n` partial slots (stride `stride` floats) of one split tile,
// for rows ra and rb of each of the H halves and of each of the NT activation
// rows this lane finishes (row j at + j * jstride; only the first `live` of
// them exist) (`base` = slot 0, half h at + h * MN): v[j][h][e] =
// (((0 + s0) + s1) + ... + s(n-1)) + v[j][h][e], slot order whatever n is. All
// loads of a chunk of CH slots are issued before the first add, so a tile
// reduced over <= CH slots costs one L2 round trip.
template <int H, int NT = 1>
__device__ __forceinline__ void sum_tile_slots(const float* base, size_t MN, size_t stride, int n, int ra, int rb,
                                               int N, size_t jstride, int live, float (&v)[NT][2][2]) {
  constexpr int CH = (16 / (H * NT)) > 1 ? 16 / (H * NT) : 1;
  float acc[NT][H][2];
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int h = 0; h < H; ++h) acc[j][h][0] = acc[j][h][1] = 0.f;
  for (int c0 = 0; c0 < n; c0 += CH) {
    float s[NT][H][2][CH];
#pragma unroll
    for (int c = 0; c < CH; ++c) {
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const bool in = c0 + c < n && j < live;
        const float* q = base + (size_t)(c0 + c) * stride + (size_t)j * jstride;
#pragma unroll
        for (int h = 0; h < H; ++h) {
          s[j][h][0][c] = (in && ra < N) ? __ldcg(q + h * MN + ra) : 0.f;
          s[j][h][1][c] = (in && rb < N) ? __ldcg(q + h * MN + rb) : 0.f;
        }
      }
    }
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      if (c0 + c < n) {
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
          for (int h = 0; h < H; ++h) {
            acc[j][h][0] += s[j][h][0][c];
            acc[j][h][1] += s[j][h][1][c];
          }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int h = 0; h < H; ++h) {
      if (ra < N) v[j][h][0] = acc[j][h][0] + v[j][h][0];
      if (rb < N) v[j][h][1] = acc[j][h][1] + v[j][h][1];
    }
}

// cp.async helpers (sm_80+ asynchronous global -> shared copies, tracked per
// thread in commit groups).
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_8(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
// 4-byte copy of which only the first `src_bytes` (1..4) are read; the rest is
// zero-filled.
__device__ __forceinline__ void cp_async_4(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// TMA and mbarrier helpers for the pair kernel.
__device__ int g_gemv_error = 0;  // a bounded wait gave up: bit 0 weight stream, bit 1 split-tile reduce
// How long a bounded wait on another CTA or on a copy lasts before it gives up
// (nanoseconds of %globaltimer). 2 s; nf4b_debug_set_wait_limit shortens it
// for the failure-detection tests. The drain after a timeout keeps its own
// fixed limit (kDrainNs), so copies still in flight always land first.
__device__ unsigned long long g_gemv_wait_ns = 2000000000ull;
constexpr unsigned long long kDrainNs = 2000000000ull;

__device__ __forceinline__ void mbar_init1(uint32_t bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// Box (x bytes, y rows) of a 2-D uint8 map into shared memory; completion
// counted on `bar`. x is a multiple of 64 (16-byte aligned as TMA requires).
__device__ __forceinline__ void tma_box(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
// Bounded wait for phase `parity` of `bar` (2 s by %globaltimer); false after
// recording the timeout in g_gemv_error. The clock is read only once the
// first probe finds the phase incomplete.
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long start = gemv_globaltimer(), limit = g_gemv_wait_ns;
  for (uint32_t i = 1;; ++i) {
    if (mbar_try(bar, parity)) return true;
    if ((i & 63u) == 0u && gemv_globaltimer() - start > limit) {
      atomicOr(&g_gemv_error, 1);
      return false;
    }
  }
}
// After a bounded wait gave up: wait for the n copies still in flight in
// stages st, st + 1, ... of an R-stage ring, so that no copy lands in shared
// memory the CTA has released - all of them within one deadline (kDrainNs
// from the start of the drain), after which the rest are not waited for.
template <int R>
__device__ __forceinline__ void drain_ring(uint32_t bar_s, int st, int n, uint32_t phase) {
  const unsigned long long deadline = gemv_globaltimer() + kDrainNs;
  for (int d = 0; d < n; ++d) {
    const int sd = (st + d) % R;
    const uint32_t bar = bar_s + 8 * sd, par = (phase >> sd) & 1u;
    for (uint32_t i = 0; !mbar_try(bar, par); ++i)
      if ((i & 63u) == 63u && gemv_globaltimer() > deadline) return;
  }
}

// Bounded wait (2 s by %globaltimer) until the global count at `ctr` reaches
// `need`, acquire; false after recording the timeout in g_gemv_error (bit 2).
__device__ __forceinline__ bool mbar_free_wait_count(const int* ctr, int need) {
  unsigned long long start = 0;
  for (uint32_t i = 0;; ++i) {
    int seen;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(seen) : "l"(ctr) : "memory");
    if (seen >= need) return true;
    if ((i & 15u) == 0u) {
      const unsigned long long now = gemv_globaltimer();
      if (i == 0) {
        start = now;
      } else if (now - start > g_gemv_wait_ns) {
        atomicOr(&g_gemv_error, 4);
        return false;
      }
    }
  }
}

// A fused wqkv store's rotary row (staged in shared memory: (cos, sin) pairs,
// 128 values) and the cache row it writes.
struct RopeKv {
  const float* f;
  long long pos;
};

// Output feature r (bf16 y) and its rotary partner r ^ 1 (yp), with the
// arithmetic of qk_rope_kv without q/k norm (app/engine/fusedlayer.py:56-92):
// a q feature rotated into rk_q, a k feature rotated into the key cache at
// pos, a v feature copied into the value cache at pos (rows outside the
// cache are not written).
__device__ __forceinline__ void rope_kv_row(const GemvParams& p, const RopeKv& rk, int r, bf16_t y, bf16_t yp) {
  const int head = r >> 7, d = r & 127;
  const int nh = p.rk_nh, nkv = p.rk_nkv;
  const bool in_cache = rk.pos >= 0 && rk.pos < p.rk_max_len;
  if (head < nh + nkv) {
    const float x = bf2f(y), xp = bf2f(yp);
    const float x0 = (d & 1) ? xp : x, x1 = (d & 1) ? x : xp;
    const float c = rk.f[d & ~1], sn = rk.f[d | 1];
    const float o = (d & 1) ? __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, sn))
                            : __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
    if (head < nh)
      p.rk_q[r] = f2bf(o);
    else if (in_cache)
      p.rk_k[((size_t)(head - nh) * p.rk_max_len + rk.pos) * 128 + d] = f2bf(o);
  } else if (in_cache) {
    p.rk_v[((size_t)(head - nh - nkv) * p.rk_max_len + rk.pos) * 128 + d] = y;
  }
}

// Both rows of a lane (ra, rb) with their partners from lane ^ 4 (row g ^ 1):
// called by the 8 lanes of activation row 0 (t == 0) together.
__device__ __forceinline__ void rope_kv_rows(const GemvParams& p, const RopeKv& rk, int ra, int rb, bf16_t ya,
                                             bf16_t yb) {
  const bf16_t pa = (bf16_t)__shfl_xor_sync(0x11111111u, (unsigned)ya, 4);
  const bf16_t pb = (bf16_t)__shfl_xor_sync(0x11111111u, (unsigned)yb, 4);
  rope_kv_row(p, rk, ra, ya, pa);
  rope_kv_row(p, rk, rb, yb, pb);
}

// Store the outputs of row tile `rt` (rows g, g + 8 of activation row t):
// the gate of the two halves for a gated pair, else the epilogue of half 0
// (and, given `rk`, the fused rotary + KV-cache write).
template <bool kGated, bool kF16 = false>
__device__ __forceinline__ void store_pair_tile(const GemvParams& p, int rt, int g, int t,
                                                const float (&v)[2][2], const RopeKv* rk = nullptr) {
  const int N = p.N;
  const int ra = rt * 16 + g, rb = ra + 8;
  if (t >= p.M) return;
  const size_t oa = (size_t)t * N + ra, ob = (size_t)t * N + rb;
  if (kGated) {
    if (ra < N) p.y[oa] = gate_bf16<kF16>(v[0][0], v[1][0]);
    if (rb < N) p.y[ob] = gate_bf16<kF16>(v[0][1], v[1][1]);
  } else if (rk != nullptr) {  // one activation row, n_out % 16 == 0 (bf16 only)
    const bf16_t ya = epilogue(v[0][0], p.epi, p.operand, oa), yb = epilogue(v[0][1], p.epi, p.operand, ob);
    p.y[oa] = ya;
    p.y[ob] = yb;
    rope_kv_rows(p, *rk, ra, rb, ya, yb);
  } else {
    if (ra < N) p.y[oa] = epilogue<kF16>(v[0][0], p.epi, p.operand, oa);
    if (rb < N) p.y[ob] = epilogue<kF16>(v[0][1], p.epi, p.operand, ob);
  }
}

// Finish row tile `rt` of the pair kernel from this warp's partial sums
// v[j][half][row g / g + 8] of activation rows t + 2j (j < NT; NT > 1 is the
// register-fed kernel's several column tiles, whose lane holds every other
// activation row). A tile inside the warp's run is stored at once (returns
// false). A split tile is published as soon as the warp's part of it is done:
// the partial goes to this warp's slot (slot = warp - first contributing
// warp) and lane 0 counts the warp in with an acquire-release atomic whose
// result (`old`, lane 0) is only looked at after the warp's run, by
// finish_tile_rows: no warp waits for another, and the last to arrive reduces
// (returns true). (Publishing every split tile only after the run was
// measured slower: the first tile's reduction then no longer overlaps the run.)
template <bool kGated, bool kF16 = false, int NT = 1>
__device__ __forceinline__ bool publish_tile_rows(const GemvParams& p, int rt, int u0, int u1, int gw, int g,
                                                  int t, int lane, const float (*v)[2][2], int& old,
                                                  const RopeKv* rk = nullptr) {
  constexpr int H = kGated ? 2 : 1;
  const int per_tile = p.blocks_per_tile * H;
  const int t0 = rt * per_tile, t1 = t0 + per_tile - 1;
  if (t0 >= u0 && t1 < u1) {
#pragma unroll
    for (int j = 0; j < NT; ++j) store_pair_tile<kGated, kF16>(p, rt, g, t + 2 * j, v[j], rk);
    return false;
  }
  const int w_lo = warp_of(t0, p.uq, p.ur);
  const int N = p.N, M = p.M;
  const int ra = rt * 16 + g, rb = ra + 8;
  const size_t MN = (size_t)M * N;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int row = t + (NT > 1 ? 2 * j : 0);
    if (row < M) {
      float* slot = p.partial + (size_t)(gw - w_lo) * H * MN + (size_t)row * N;
#pragma unroll
      for (int h = 0; h < H; ++h) {
        if (ra < N) __stcg(slot + h * MN + ra, v[j][h][0]);
        if (rb < N) __stcg(slot + h * MN + rb, v[j][h][1]);
      }
    }
  }
  // The warp barrier orders every lane's partial before lane 0's release.
  __syncwarp();
  if (lane == 0) old = atomic_add_acq_rel(p.counters + rt, 1);
  return true;
}

template <bool kGated, bool kF16 = false>
__device__ __forceinline__ bool publish_pair_tile(const GemvParams& p, int rt, int u0, int u1, int gw, int g,
                                                  int t, int lane, const float (&v)[2][2], int& old,
                                                  const RopeKv* rk = nullptr) {
  return publish_tile_rows<kGated, kF16, 1>(p, rt, u0, u1, gw, g, t, lane, &v, old, rk);
}

// After the warp's run: if it was the last of split tile rt's contributors to
// arrive, sum every slot in slot order, (((0 + s0) + s1) + ...), and store -
// the residual or gate operand is fetched in the same round trip as the
// slots - then re-zero the counter for the next launch. Rows as
// publish_tile_rows.
template <bool kGated, bool kF16 = false, int NT = 1>
__device__ __forceinline__ void finish_tile_rows(const GemvParams& p, int rt, int old, int g, int t, int lane,
                                                 const RopeKv* rk = nullptr) {
  constexpr int H = kGated ? 2 : 1;
  constexpr int JS = NT > 1 ? 2 : 0;  // activation-row step between column tiles
  const int per_tile = p.blocks_per_tile * H;
  const int t0 = rt * per_tile;
  const int n = warp_of(t0 + per_tile - 1, p.uq, p.ur) - warp_of(t0, p.uq, p.ur) + 1;
  old = __shfl_sync(0xffffffffu, old, 0);  // lane 0's acquire; the shuffle orders the lanes' reads after it
  if (old != n - 1) return;
  const int N = p.N, M = p.M;
  const int ra = rt * 16 + g, rb = ra + 8;
  const size_t MN = (size_t)M * N;
  if (lane == 0) p.counters[rt] = 0;
  if (t >= M) return;
  const int live = NT > 1 ? (M - t + 1) / 2 : 1;  // rows t, t + 2, ... below M
  const bool opnd = !kGated && p.epi != NF4B_EPI_NONE;
  uint16_t opa[NT], opb[NT];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const size_t oa = (size_t)(t + JS * j) * N + ra, ob = (size_t)(t + JS * j) * N + rb;
    const bool in = opnd && j < live;
    opa[j] = (in && ra < N) ? __ldcg(p.operand + oa) : (uint16_t)0;
    opb[j] = (in && rb < N) ? __ldcg(p.operand + ob) : (uint16_t)0;
  }
  float v[NT][2][2];
#pragma unroll
  for (int j = 0; j < NT; ++j) v[j][0][0] = v[j][0][1] = v[j][1][0] = v[j][1][1] = 0.f;
  sum_tile_slots<H, NT>(p.partial + (size_t)t * N, MN, H * MN, n, ra, rb, N, (size_t)JS * N, live, v);
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    if (j >= live) break;
    const size_t oa = (size_t)(t + JS * j) * N + ra, ob = (size_t)(t + JS * j) * N + rb;
    if (kGated) {
      if (ra < N) p.y[oa] = gate_bf16<kF16>(v[j][0][0], v[j][1][0]);
      if (rb < N) p.y[ob] = gate_bf16<kF16>(v[j][0][1], v[j][1][1]);
    } else if (rk != nullptr) {  // one activation row, n_out % 16 == 0 (bf16 only)
      const bf16_t ya = epilogue_value(v[j][0][0], p.epi, bf2f(opa[j]));
      const bf16_t yb = epilogue_value(v[j][0][1], p.epi, bf2f(opb[j]));
      p.y[oa] = ya;
      p.y[ob] = yb;
      rope_kv_rows(p, *rk, ra, rb, ya, yb);
    } else {
      if (ra < N) p.y[oa] = epilogue_value<kF16>(v[j][0][0], p.epi, act2f<kF16>(opa[j]));
      if (rb < N) p.y[ob] = epilogue_value<kF16>(v[j][0][1], p.epi, act2f<kF16>(opb[j]));
    }
  }
}

template <bool kGated, bool kF16 = false>
__device__ __forceinline__ void finish_split_tile(const GemvParams& p, int rt, int old, int g, int t, int lane,
                                                  const RopeKv* rk = nullptr) {
  finish_tile_rows<kGated, kF16, 1>(p, rt, old, g, t, lane, rk);
}

// A warp that gave up on a wait while computing unit tile `rt_now` of its run
// [u0, u1) still counts itself into the split tiles it has not published (the
// current one and the run's last), with zero partial sums, so every tile
// counter returns to zero after the last contributor's reduction and the
// caller's workspace stays reusable. The outputs of such a call are invalid;
// nf4b_device_error reports it.
template <bool kGated>
__device__ __forceinline__ void abort_split_tiles(const GemvParams& p, int rt_now, int u0, int u1, int gw, int g,
                                                  int t, int lane, int& split_a, int& old_a, int& split_b,
                                                  int& old_b) {
  const int per_tile = p.blocks_per_tile * (kGated ? 2 : 1);
  const int rt_last = (u1 - 1) / per_tile;
  const float zero[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
  for (int rt = rt_now; rt <= rt_last; rt += (rt_last > rt_now ? rt_last - rt_now : 1)) {
    const int t0 = rt * per_tile;
    if (t0 >= u0 && t0 + per_tile - 1 < u1) continue;  // a whole tile: nobody waits on it
    int old = 0;
    publish_pair_tile<kGated>(p, rt, u0, u1, gw, g, t, lane, zero, old);
    if (split_a < 0) {
      split_a = rt;
      old_a = old;
    } else {
      split_b = rt;
      old_b = old;
    }
  }
}

// Pair kernel. A unit is 16 weight rows x SU * 128 codes (SU = 2 for
// blocksize-64 weights with k_in % 256 == 0, else 1). Units are numbered
// tile-major; within a tile, the k units of W and then (gated pair) those of
// W3, so one warp run covers both halves of a tile where it can and the
// finisher sees both.
//
// Each warp streams its run through a private ring of R = 6 / SU stages,
// R - 1 units ahead. Lane 0 requests a unit's 16 rows x SU * 64 bytes as one
// TMA box (completion on the stage's mbarrier); lanes t = 0 and t = 1 copy the
// scale data of rows g and g + 8 with cp.async (one commit group per unit,
// released by `cp.async.wait_group R-1`). A box lands row-major, so lane (g, t)
// reads the 16 bytes of rows g and g + 8 it multiplies for each 128-code
// sub-unit, and every 8-lane phase of those 128-bit loads covers 128
// contiguous bytes (no bank conflicts) when SU = 1, 2-way when SU = 2.
//
// Scale data per row and unit (8 * SU bytes): nested - the 4-byte aligned
// window(s) holding the unit's 8-bit codes, then one second-level scale per
// 128-code sub-unit (its two 64-blocks share it); plain - the fp32 scales of
// the unit's blocks.
template <bool kGated, int SU>
__global__ void __launch_bounds__(GEMV_PAIR_WARPS * 32, 1)
    nf4_gemv_pair_kernel(const __grid_constant__ GemvParams p) {
  constexpr int R = GEMV_PAIR_STAGE_KB / SU;
  constexpr int WB = 1024 * SU;  // weight bytes per stage
  constexpr int SB = 128 * SU;   // scale bytes per stage
  static_assert(R >= 2, "ring too short");
  constexpr int kT = GEMV_PAIR_WARPS * 32;
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ double norm_red[GEMV_PAIR_WARPS];
  const uint8_t* lut = smem;
  const float* code2_s = reinterpret_cast<const float*>(smem + GEMV_LUT_BYTES);
  const float* code2_s3 = code2_s + 256;
  const uint8_t* xs = smem + GEMV_PAIR_X_OFFSET;

  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;  // warp in block
  const int gw = blockIdx.x * GEMV_PAIR_WARPS + wib;
  const bool active = gw < p.warps_total;
  const int u0 = active ? gw * p.uq + min(gw, p.ur) : 0;
  const int u1 = active ? u0 + p.uq + (gw < p.ur ? 1 : 0) : 0;
  const int g = lane >> 2, t = lane & 3;
  const int B = p.blocks_per_tile;  // units per row tile and half
  const int per_tile = kGated ? 2 * B : B;
  const int N = p.N, K = p.K, M = p.M;
  const uint32_t lane_base = (uint32_t)lane * 4u;
  const int bs_shift = p.bs_shift;
  const bool bs64 = bs_shift == 6;
  const int nblk = K >> bs_shift;  // scale blocks per weight row
  const long long a8_total = (long long)N * nblk;

  const uint8_t* wring = smem + GEMV_PAIR_W_OFFSET + wib * (R * WB);
  const uint8_t* sring = smem + GEMV_PAIR_SC_OFFSET + wib * (R * SB);
  const uint32_t wring_s = smem_addr(wring), sring_s = smem_addr(sring);
  const uint32_t bar_s = smem_addr(smem + GEMV_PAIR_BAR_OFFSET + wib * (R * 8));
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < R; ++i) mbar_init1(bar_s + 8 * i);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();

  // Load cursor: tile lt, half lh, k unit lk (incremental, no divisions).
  int lt = u0 / per_tile, lk = u0 - lt * per_tile, lh = 0;
  if (kGated && lk >= B) {
    lh = 1;
    lk -= B;
  }
  int ct = lt, ch = lh, ck = lk;

  // Scale arrays of the tile/half being loaded; lanes t = 0 and t = 1 copy the
  // scales of row g and g + 8 respectively (`sbase` = that row's first block).
  const uint8_t* a8 = p.a8;
  const float* absmax = p.absmax;
  long long sbase = 0;
  auto set_rows = [&](int rt, int h) {
    sbase = (long long)min(rt * 16 + g + 8 * t, N - 1) * nblk;
    a8 = (kGated && h) ? p.a8_3 : p.a8;
    absmax = (kGated && h) ? p.absmax3 : p.absmax;
  };
  set_rows(lt, lh);
  auto step_load = [&]() {
    if (++lk == B) {
      lk = 0;
      if (kGated && lh == 0) {
        lh = 1;
      } else {
        lh = 0;
        ++lt;
      }
      set_rows(lt, lh);
    }
  };
  // Request the load cursor's unit into stage `st`.
  auto issue = [&](int st) {
    if (lane == 0) {
      const uint32_t bar = bar_s + 8 * st;
      mbar_expect(bar, (uint32_t)WB);
      // rows past n_out read as zeros (TMA bounds); their outputs are never stored
      tma_box(wring_s + st * WB, (kGated && lh) ? &p.wmap3 : &p.wmap, lk * 64 * SU, lt * 16, bar);
    }
    if (t < 2) {
      const uint32_t ds = sring_s + st * SB + (g + 8 * t) * (8 * SU);
      const long long be = sbase + ((lk * 128 * SU) >> bs_shift);
      if (SU == 2) {
        // k_in % 256 == 0, so a unit's four blocks start at a multiple of 4:
        // nested - their codes are one aligned word and (second-level blocks
        // of >= 4) share one second-level scale; plain - 16 aligned bytes.
        if (p.nested) {
          cp_async_4(ds, a8 + be, 4u);
          cp_async_4(ds + 4, absmax + (be >> p.bs2_shift), 4u);
        } else {
          cp_async_16(ds, absmax + be);
        }
      } else if (p.nested) {
        // the 4-byte aligned window holding this unit's one or two 8-bit codes
        const long long w0 = be & ~3LL;
        const long long left = a8_total - w0;
        cp_async_4(ds, a8 + w0, (uint32_t)(left < 4 ? left : 4));
        cp_async_4(ds + 4, absmax + (be >> p.bs2_shift), 4u);
      } else if (bs64) {
        cp_async_8(ds, absmax + be);
      } else {
        cp_async_4(ds, absmax + be, 4u);
        cp_async_4(ds + 4, absmax + be, 4u);
      }
    }
  };
  // Compute cursor and the byte phase (row * nblk) & 3 of rows g and g+8
  // within their 4-byte scale-code windows.
  int ph_a = 0, ph_b = 0;
  auto set_phase = [&](int rt) {
    ph_a = (int)(((long long)min(rt * 16 + g, N - 1) * nblk) & 3);
    ph_b = (int)(((long long)min(rt * 16 + g + 8, N - 1) * nblk) & 3);
  };
  set_phase(ct);

  // The nested scales' code2 tables (1 KB each) are copied asynchronously as
  // the first commit group, so the table build below never waits on memory.
  if (p.nested) {
    if (threadIdx.x < 64) {
      cp_async_16(smem_addr(smem + GEMV_LUT_BYTES) + threadIdx.x * 16, p.code2 + threadIdx.x * 4);
    } else if (kGated && threadIdx.x < 128) {
      const int i = threadIdx.x - 64;
      cp_async_16(smem_addr(smem + GEMV_LUT_BYTES + 1024) + i * 16, p.code2_3 + i * 4);
    }
  }
  cp_async_commit();
  // Prologue: R - 1 units requested (one cp.async group each, empty past the run).
#pragma unroll
  for (int i = 0; i < R - 1; ++i) {
    if (u0 + i < u1) {
      issue(i);
      step_load();
    }
    cp_async_commit();
  }
  // The pair table is built while the first units are in flight.
  build_pair_lut<kT>(smem);
  pdl_launch_dependents();
  if (active && NF4B_GEMV_PREFETCH_EARLY) prefetch_next(p, gw, lane);
  pdl_wait();
  // x, written by earlier work on the stream, is staged once per CTA so that
  // no unit waits on an L2 round trip for its slice of it.
  if (p.x_staged) {
    const int n16 = (M * K) >> 3;
    const uint4* src = reinterpret_cast<const uint4*>(p.x);
    uint4* dst = reinterpret_cast<uint4*>(smem + GEMV_PAIR_X_OFFSET);
    for (int i = threadIdx.x; i < n16; i += kT) dst[i] = __ldcg(src + i);
  }
  cp_async_wait<R - 1>();  // this thread's code2 copy (R - 1 unit groups were committed after it)
  __syncthreads();         // the pair table, code2 and x are visible to every warp
  // the fused RMSNorm (x is staged whenever it is requested)
  if (p.norm_w != nullptr)
    rms_normalise_staged<kT>(reinterpret_cast<uint16_t*>(smem + GEMV_PAIR_X_OFFSET), M, K, p.norm_w, p.norm_eps,
                             norm_red);

  // x: column c of the MMA is (activation row c >> 1, block parity c & 1);
  // lane (g, t) supplies column g for codes of block parity t >> 1.
  const int xtok = g >> 1;
  const bool xlane = (xtok < M) && ((g & 1) == (t >> 1));
  const size_t xrow_off = (size_t)(xlane ? xtok : 0) * K * 2 + t * 64;  // bytes
  const uint4* xrow = reinterpret_cast<const uint4*>(
      (p.x_staged ? xs : reinterpret_cast<const uint8_t*>(p.x)) + xrow_off);
  const uint4* xrow_s = reinterpret_cast<const uint4*>(xs + xrow_off);

  float acc_a = 0.f, acc_b = 0.f;    // W (or W1): rows g, g+8 for activation row t
  float acc3_a = 0.f, acc3_b = 0.f;  // gated pair: W3
  // split tiles this warp published (at most two: its run's first and last)
  int split_a = -1, split_b = -1, old_a = 0, old_b = 0;
  int st_use = 0, st_fill = R - 1;
  uint32_t phase = 0;  // bit s: parity of stage s's next completion
  for (int u = u0; u < u1; ++u) {
    // Request unit u + R - 1 into the stage computed last iteration (the warp
    // barrier orders every lane's reads of it before the overwrite).
    __syncwarp();
    if (u + R - 1 < u1) {
      issue(st_fill);
      step_load();
    }
    cp_async_commit();
    st_fill = st_fill + 1 == R ? 0 : st_fill + 1;
    cp_async_wait<R - 1>();  // unit u's scales (this lane's copies)
    if (!mbar_wait_bounded(bar_s + 8 * st_use, (phase >> st_use) & 1u)) {
      drain_ring<R>(bar_s, st_use, min(R, u1 - u), phase);  // units u .. u + R - 1 were requested
      abort_split_tiles<kGated>(p, ct, u0, u1, gw, g, t, lane, split_a, old_a, split_b, old_b);
      break;
    }
    phase ^= 1u << st_use;
    __syncwarp();            // every lane's scale copies are visible
    const uint8_t* wst = wring + st_use * WB;
    const uint8_t* sst = sring + st_use * SB;
    st_use = st_use + 1 == R ? 0 : st_use + 1;

    const int rt = ct, kb = ck, hh = ch;
    const int pha = ph_a, phb = ph_b;
    if (++ck == B) {
      ck = 0;
      if (kGated && ch == 0) {
        ch = 1;
      } else {
        ch = 0;
        ++ct;
        set_phase(ct);
      }
    }

    // Scale data of rows g and g + 8 for this unit.
    uint32_t sa[2 * SU], sb[2 * SU];
    if (SU == 2) {
      const uint4 va = *reinterpret_cast<const uint4*>(sst + g * 16);
      const uint4 vb = *reinterpret_cast<const uint4*>(sst + (g + 8) * 16);
      sa[0] = va.x; sa[1] = va.y; sa[2 % (2 * SU)] = va.z; sa[3 % (2 * SU)] = va.w;
      sb[0] = vb.x; sb[1] = vb.y; sb[2 % (2 * SU)] = vb.z; sb[3 % (2 * SU)] = vb.w;
    } else {
      const uint2 va = *reinterpret_cast<const uint2*>(sst + g * 8);
      const uint2 vb = *reinterpret_cast<const uint2*>(sst + (g + 8) * 8);
      sa[0] = va.x; sa[1] = va.y;
      sb[0] = vb.x; sb[1] = vb.y;
    }
    float ya = 0.f, yb = 0.f;
#pragma unroll
    for (int i = 0; i < SU; ++i) {
      const int kb2 = kb * SU + i;  // 128-code sub-unit index within the row
      float se_a, so_a, se_b, so_b;
      if (p.nested) {
        const float* c2 = (kGated && hh) ? code2_s3 : code2_s;
        const float off = (kGated && hh) ? p.offset3 : p.offset;
        uint32_t ea, oa, eb, ob;
        float s2a, s2b;
        if (SU == 2) {
          // blocks 2i, 2i+1 of the unit are bytes 2i, 2i+1 of the code word
          ea = (sa[0] >> (16 * i)) & 0xFFu;
          oa = (sa[0] >> (16 * i + 8)) & 0xFFu;
          eb = (sb[0] >> (16 * i)) & 0xFFu;
          ob = (sb[0] >> (16 * i + 8)) & 0xFFu;
          s2a = __uint_as_float(sa[1]);
          s2b = __uint_as_float(sb[1]);
        } else {
          // the unit's first block sits at byte (row phase + block index) & 3 of the window
          const int be0 = (kb2 * 128) >> bs_shift;
          const uint32_t sha = (uint32_t)((pha + be0) & 3) * 8, shb = (uint32_t)((phb + be0) & 3) * 8;
          ea = (sa[0] >> sha) & 0xFFu;
          eb = (sb[0] >> shb) & 0xFFu;
          oa = bs64 ? (sa[0] >> (sha + 8)) & 0xFFu : ea;
          ob = bs64 ? (sb[0] >> (shb + 8)) & 0xFFu : eb;
          s2a = __uint_as_float(sa[1]);
          s2b = __uint_as_float(sb[1]);
        }
        se_a = nested_scale(c2[ea], s2a, off);
        so_a = nested_scale(c2[oa], s2a, off);
        se_b = nested_scale(c2[eb], s2b, off);
        so_b = nested_scale(c2[ob], s2b, off);
      } else {
        se_a = __uint_as_float(sa[(2 * i) % (2 * SU)]); so_a = __uint_as_float(sa[(2 * i + 1) % (2 * SU)]);
        se_b = __uint_as_float(sb[(2 * i) % (2 * SU)]); so_b = __uint_as_float(sb[(2 * i + 1) % (2 * SU)]);
      }
      uint4 xv[4];
      if (xlane) {  // SU = 2: x is always staged (shared loads); SU = 1: staged or global
        const uint4* xr = SU == 2 ? xrow_s : xrow;
#pragma unroll
        for (int j = 0; j < 4; ++j) xv[j] = xr[kb2 * 16 + j];
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) xv[j] = make_uint4(0, 0, 0, 0);
      }
      const uint4 wav = *reinterpret_cast<const uint4*>(wst + g * (64 * SU) + i * 64 + t * 16);
      const uint4 wbv = *reinterpret_cast<const uint4*>(wst + (g + 8) * (64 * SU) + i * 64 + t * 16);
      // Two independent MMA chains (even and odd k steps).
      float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
      const uint32_t wa[4] = {wav.x, wav.y, wav.z, wav.w};
      const uint32_t wb[4] = {wbv.x, wbv.y, wbv.z, wbv.w};
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const uint32_t w0 = wa[s >> 1], w1 = wb[s >> 1];
        const int j0 = 2 * (s & 1);
        const uint32_t a0 = lut_lookup(lut, w0, lut_sel(j0), lane_base);
        const uint32_t a2 = lut_lookup(lut, w0, lut_sel(j0 + 1), lane_base);
        const uint32_t a1 = lut_lookup(lut, w1, lut_sel(j0), lane_base);
        const uint32_t a3 = lut_lookup(lut, w1, lut_sel(j0 + 1), lane_base);
        const uint4& xq = xv[s >> 1];
        const uint32_t b0 = (s & 1) ? xq.z : xq.x;
        const uint32_t b1 = (s & 1) ? xq.w : xq.y;
        if (s & 1)
          mma_bf16_16816(d1, a0, a1, a2, a3, b0, b1);
        else
          mma_bf16_16816(d0, a0, a1, a2, a3, b0, b1);
      }
      // d[0] = (row g, col 2t) = even block, d[1] = odd block; d[2]/d[3] for row g+8.
      ya += fmaf(so_a, d0[1] + d1[1], (d0[0] + d1[0]) * se_a);
      yb += fmaf(so_b, d0[3] + d1[3], (d0[2] + d1[2]) * se_b);
    }
    if (kGated && hh) {
      acc3_a += ya;
      acc3_b += yb;
    } else {
      acc_a += ya;
      acc_b += yb;
    }
    if ((kb == B - 1 && (!kGated || hh == 1)) || u == u1 - 1) {
      const float v[2][2] = {{acc_a, acc_b}, {acc3_a, acc3_b}};
      int old = 0;
      if (publish_pair_tile<kGated>(p, rt, u0, u1, gw, g, t, lane, v, old)) {
        if (split_a < 0) {
          split_a = rt;
          old_a = old;
        } else {
          split_b = rt;
          old_b = old;
        }
      }
      acc_a = acc_b = acc3_a = acc3_b = 0.f;
    }
  }
  if (split_a >= 0) finish_split_tile<kGated>(p, split_a, old_a, g, t, lane);
  if (split_b >= 0) finish_split_tile<kGated>(p, split_b, old_b, g, t, lane);
  cp_async_wait<0>();
  if (!NF4B_GEMV_PREFETCH_EARLY) prefetch_next(p, gw, lane);
}

// A 16-byte shared-memory load into v when `pred`; v keeps its value otherwise
// (the destination registers are read-write, so no zero-fill is issued).
__device__ __forceinline__ void ld_shared_u4_if(bool pred, uint32_t addr, uint4& v) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t@p ld.shared.v4.u32 {%0, %1, %2, %3}, [%5];\n\t}"
      : "+r"(v.x), "+r"(v.y), "+r"(v.z), "+r"(v.w)
      : "r"((int)pred), "r"(addr));
}

// ---------------------------------------------------------------------------
// register-fed pair kernel: units of 16 rows x 256 codes, activation rows <= 8
// ---------------------------------------------------------------------------
//
// The decode case (1..8 activation rows, blocksize 64, k_in % 256 == 0). The
// units, runs and the split-tile protocol are the pair kernel's (SU = 2), but
// the weights skip shared memory: lane (g, t) loads 64-block t of the unit for
// rows g and g + 8 with one 256-bit load each straight into registers, three
// units in flight per warp (two with several column tiles). Shared memory then
// carries only the pair table, the scale codes' code2 values and x, which is
// what bounds the pair kernel's consumer (its TMA ring costs a shared-memory
// write and a read per weight byte).
//
// MMA columns are (activation row, block): column 4m + b of column tile j
// carries x of row 2j + m over block b of the unit, so one MMA chain per tile
// keeps the unit's four block sums apart and each gets its own scale after the
// unit. Lane (g, t) holds columns 2t and 2t + 1 of every tile - activation
// rows 2j + (t >> 1), blocks 2(t & 1) and 2(t & 1) + 1 - and supplies x for
// column g (row 2j + (g >> 2), block g & 3) when g & 3 == t. Lanes t and t ^ 1
// hold a row's two half-sums; they are added when a tile is finished. NT = 1,
// 2, 4 column tiles serve 1-2, 3-4 and 5-8 rows: the weights are decoded once
// (the pair-table lookups are the same) whatever the row count.
//
// Shared memory: the pair table (entry e's 32 per-lane copies at e * 256), the
// code2 value of scale code e at e * 256 + 128 + 4 * (2g + (t & 1)) (16 copies,
// so a warp's lookups never conflict; W3's at + 192), then x, rows of k_in * 2
// bytes, each 64-block's eight 16-byte chunks rotated: chunk c of block b of
// row m sits at chunk (c + (b & 3) + 4 (m & 1)) & 7 of the block's 128 bytes,
// so the eight x lanes of a load (four blocks, two rows) hit eight different
// bank groups with no padding (rows * k_in * 2 <= GEMV_REG_X_MAX).
// kRope: the fused rotary + KV-cache store of a wqkv projection (one
// activation row, not gated, bf16). kF16: fp16 activations and outputs (the
// pair table holds fp16 code pairs and the MMA is f16 x f16).
template <bool kGated, bool kNested, bool kRope = false, bool kF16 = false, int NT = 1>
__global__ void __launch_bounds__(GEMV_PAIR_WARPS * 32, 1)
    nf4_gemv_reg_kernel(const __grid_constant__ GemvParams p) {
  constexpr int kT = GEMV_PAIR_WARPS * 32;
  constexpr int kDepth = NT == 1 ? kRegDepth : 2;  // units in flight per warp
  constexpr int CH = NT == 1 ? 2 : 1;              // MMA chains per column tile
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ double norm_red[GEMV_PAIR_WARPS];
  __shared__ float rk_f[kRope ? 128 : 1];  // kRope: this token's rotary row
  static_assert(!(kRope && kGated), "the fused rotary store serves a plain projection");
  static_assert(!(kRope && (kF16 || NT > 1)), "the fused rotary store is bf16, one row");
  static_assert(NT == 1 || NT == 2 || NT == 4, "1, 2 or 4 column tiles");
  const uint8_t* lut = smem;
  uint8_t* xs = smem + GEMV_LUT_BYTES;

  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * GEMV_PAIR_WARPS + (threadIdx.x >> 5);
  const bool active = gw < p.warps_total;
  const int u0 = active ? gw * p.uq + min(gw, p.ur) : 0;
  const int u1 = active ? u0 + p.uq + (gw < p.ur ? 1 : 0) : 0;
  const int g = lane >> 2, t = lane & 3;
  const int B = p.blocks_per_tile;  // 256-code units per row tile and half
  const int per_tile = kGated ? 2 * B : B;
  const int N = p.N, K = p.K, M = p.M;
  const int nblk = K >> 6;  // 64-blocks per weight row
  const int bs2 = p.bs2_shift;
  constexpr bool nested = kNested;
  const int xrow = K * 2;

  // Load cursor: tile lt, half lh, unit lk; rows past n_out re-read row
  // n_out - 1 (their outputs are never stored).
  int lt = u0 / per_tile, lk = u0 - lt * per_tile, lh = 0;
  if (kGated && lk >= B) {
    lh = 1;
    lk -= B;
  }
  int ct = lt, ck = lk, ch = lh;
  // first 64-block of rows g and g + 8 (n_out * k_in / 64 < 2^31 is checked on the host)
  int oa = 0, ob = 0;
  auto set_rows = [&](int rt) {
    oa = min(rt * 16 + g, N - 1) * nblk;
    ob = min(rt * 16 + g + 8, N - 1) * nblk;
  };
  set_rows(lt);
  auto load = [&](RegSlot& s) {
    const uint8_t* pw = (kGated && lh) ? p.packed3 : p.packed;
    const uint8_t* pq = (kGated && lh) ? p.a8_3 : p.a8;
    const float* ps = (kGated && lh) ? p.absmax3 : p.absmax;
    const int ba = oa + lk * 4, bb = ob + lk * 4;  // the unit's first block in rows g, g + 8
    ld_stream_u8(pw + (size_t)ba * 32 + t * 32, s.wa);
    ld_stream_u8(pw + (size_t)bb * 32 + t * 32, s.wb);
    if (nested) {
      s.qa = __ldg(reinterpret_cast<const uint32_t*>(pq + ba));
      s.qb = __ldg(reinterpret_cast<const uint32_t*>(pq + bb));
      s.sa = __float_as_uint(__ldg(ps + (ba >> bs2)));
      s.sb = __float_as_uint(__ldg(ps + (bb >> bs2)));
    } else {
      const float2 fa = __ldg(reinterpret_cast<const float2*>(ps + ba + 2 * (t & 1)));
      const float2 fb = __ldg(reinterpret_cast<const float2*>(ps + bb + 2 * (t & 1)));
      s.qa = __float_as_uint(fa.x);
      s.sa = __float_as_uint(fa.y);
      s.qb = __float_as_uint(fb.x);
      s.sb = __float_as_uint(fb.y);
    }
    if (++lk == B) {
      lk = 0;
      if (kGated && lh == 0) {
        lh = 1;
      } else {
        lh = 0;
        ++lt;
        set_rows(lt);
      }
    }
  };

  RegSlot sl[kDepth];
#pragma unroll
  for (int d = 0; d < kDepth; ++d)
    if (u0 + d < u1) load(sl[d]);

  // The pair table, built while the first units are in flight; the code2
  // values are requested now and their copies stored after the dependency
  // wait, so no thread reaches the wait behind a global load.
  float c2v[2048 / kT];
  if (nested) load_code2_copies<kT>(p.code2, kGated ? p.code2_3 : nullptr, c2v);
  build_pair_lut_fast<kT, kF16>(smem);
  pdl_launch_dependents();
  pdl_wait();
  if (nested) store_code2_copies<kT>(smem, c2v);
  // kRope: the rotary row and the cache position (both written before this
  // launch) are requested with x and stored after x's loads are out.
  long long rk_pos = 0;
  float rk_val = 0.f;
  if (kRope) {
    if (threadIdx.x < 128) rk_val = load_freq(p.rk_freqs, threadIdx.x, p.rk_ftype);
    rk_pos = p.rk_pos[0];
  }
  // x, written by earlier work on the stream, staged in the rotated layout:
  // x is [M, k_in] contiguous, so the rows form one run of 16-byte chunks,
  // and each thread issues up to 8 of its chunks' loads before storing any
  // (one L2 round trip per 8 x 8 KB instead of one per row).
  {
    constexpr int kBatch = 8;
    const int n16 = K >> 3, total = M * n16;
    const uint4* src = reinterpret_cast<const uint4*>(p.x);
    for (int base = threadIdx.x; base < total; base += kBatch * kT) {
      uint4 v[kBatch];
#pragma unroll
      for (int b = 0; b < kBatch; ++b)
        if (base + b * kT < total) v[b] = __ldcg(src + base + b * kT);
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int i = base + b * kT;
        if (i < total) {
          const int m = i / n16, c = i - m * n16;
          const int blk = c >> 3, rot = ((c & 7) + (blk & 3) + 4 * (m & 1)) & 7;
          *reinterpret_cast<uint4*>(xs + m * xrow + blk * 128 + rot * 16) = v[b];
        }
      }
    }
  }
  if (kRope && threadIdx.x < 128) rk_f[threadIdx.x] = rk_val;
  __syncthreads();
  if (p.norm_w != nullptr)
    rms_normalise_staged<kT, 2, kF16>(reinterpret_cast<uint16_t*>(xs), M, K, p.norm_w, p.norm_eps, norm_red,
                                      xrow / 2);

  const uint32_t lane_base = (uint32_t)lane * 4u;
  const uint32_t c2_base = 128u + (uint32_t)(2 * g + (t & 1)) * 4u;
  const uint32_t qsel0 = 0x5504u | ((uint32_t)(2 * (t & 1)) << 4);
  const uint32_t qsel1 = 0x5504u | ((uint32_t)(2 * (t & 1) + 1) << 4);
  // x lane: block t of rows 2j + (g >> 2); its chunks are rotated by xrot.
  const bool xsup = (g & 3) == t;
  const int xr0 = g >> 2;
  const uint32_t xrot = (uint32_t)(t + 4 * xr0);
  const uint32_t xb_s = smem_addr(xs + xr0 * xrow + t * 128);
  // Lanes that supply no x for tile j keep zeros in its B registers: the
  // loads are predicated, so the zeros are written once.
  bool xld[NT];
  uint4 xq[NT];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    xld[j] = xsup && 2 * j + xr0 < M;
    xq[j] = make_uint4(0, 0, 0, 0);
  }
  const int tok = (t & 1) ? 64 : (t >> 1);  // the first activation row this lane publishes (64: none)

  float acc_a[NT], acc_b[NT];    // W (or W1): rows g, g + 8 of activation rows tok + 2j
  float acc3_a[NT], acc3_b[NT];  // gated pair: W3
#pragma unroll
  for (int j = 0; j < NT; ++j) acc_a[j] = acc_b[j] = acc3_a[j] = acc3_b[j] = 0.f;
  int split_a = -1, split_b = -1, old_a = 0, old_b = 0;
  auto compute = [&](const RegSlot& s, int u) {
    const int rt = ct, kb = ck, hh = ch;
    if (++ck == B) {
      ck = 0;
      if (kGated && ch == 0) {
        ch = 1;
      } else {
        ch = 0;
        ++ct;
      }
    }
    float s0a, s1a, s0b, s1b;
    if (nested) {
      const uint32_t cb = c2_base + ((kGated && hh) ? 64u : 0u);
      const float off = (kGated && hh) ? p.offset3 : p.offset;
      const float s2a = __uint_as_float(s.sa), s2b = __uint_as_float(s.sb);
      s0a = nested_scale(*reinterpret_cast<const float*>(lut + __byte_perm(s.qa, cb, qsel0)), s2a, off);
      s1a = nested_scale(*reinterpret_cast<const float*>(lut + __byte_perm(s.qa, cb, qsel1)), s2a, off);
      s0b = nested_scale(*reinterpret_cast<const float*>(lut + __byte_perm(s.qb, cb, qsel0)), s2b, off);
      s1b = nested_scale(*reinterpret_cast<const float*>(lut + __byte_perm(s.qb, cb, qsel1)), s2b, off);
    } else {
      s0a = __uint_as_float(s.qa);
      s1a = __uint_as_float(s.sa);
      s0b = __uint_as_float(s.qb);
      s1b = __uint_as_float(s.sb);
    }
    // NT == 1: two independent MMA chains (even and odd k steps); several
    // column tiles are independent chains already. x of a tile: one 16-byte
    // chunk (8 codes) per two steps.
    float d[NT][CH][4];
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int c = 0; c < CH; ++c) d[j][c][0] = d[j][c][1] = d[j][c][2] = d[j][c][3] = 0.f;
    const uint32_t xu = xb_s + (uint32_t)kb * 512u;
#pragma unroll
    for (int st = 0; st < 16; ++st) {
      if ((st & 1) == 0) {
        const uint32_t off = (((uint32_t)(st >> 1) + xrot) & 7u) * 16u;
#pragma unroll
        for (int j = 0; j < NT; ++j) ld_shared_u4_if(xld[j], xu + (uint32_t)(2 * j * xrow) + off, xq[j]);
      }
      const uint32_t w0 = s.wa[st >> 1], w1 = s.wb[st >> 1];
      const int j0 = 2 * (st & 1);
      const uint32_t a0 = lut_lookup(lut, w0, lut_sel(j0), lane_base);
      const uint32_t a2 = lut_lookup(lut, w0, lut_sel(j0 + 1), lane_base);
      const uint32_t a1 = lut_lookup(lut, w1, lut_sel(j0), lane_base);
      const uint32_t a3 = lut_lookup(lut, w1, lut_sel(j0 + 1), lane_base);
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const uint32_t b0 = (st & 1) ? xq[j].z : xq[j].x;
        const uint32_t b1 = (st & 1) ? xq[j].w : xq[j].y;
        mma_act<kF16>(d[j][CH == 2 ? (st & 1) : 0], a0, a1, a2, a3, b0, b1);
      }
    }
    // d[.][0] = (row g, block 2(t & 1)), d[.][1] = its successor; d[.][2], d[.][3] for row g + 8.
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      float e0 = d[j][0][0], e1 = d[j][0][1], e2 = d[j][0][2], e3 = d[j][0][3];
      if (CH == 2) {
        e0 += d[j][CH - 1][0];
        e1 += d[j][CH - 1][1];
        e2 += d[j][CH - 1][2];
        e3 += d[j][CH - 1][3];
      }
      const float ya = fmaf(s1a, e1, e0 * s0a);
      const float yb = fmaf(s1b, e3, e2 * s0b);
      if (kGated && hh) {
        acc3_a[j] += ya;
        acc3_b[j] += yb;
      } else {
        acc_a[j] += ya;
        acc_b[j] += yb;
      }
    }
    if ((kb == B - 1 && (!kGated || hh == 1)) || u == u1 - 1) {
      float v[NT][2][2];
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        v[j][0][0] = acc_a[j] + __shfl_xor_sync(0xffffffffu, acc_a[j], 1);
        v[j][0][1] = acc_b[j] + __shfl_xor_sync(0xffffffffu, acc_b[j], 1);
        if (kGated) {
          v[j][1][0] = acc3_a[j] + __shfl_xor_sync(0xffffffffu, acc3_a[j], 1);
          v[j][1][1] = acc3_b[j] + __shfl_xor_sync(0xffffffffu, acc3_b[j], 1);
        } else {
          v[j][1][0] = v[j][1][1] = 0.f;
        }
        acc_a[j] = acc_b[j] = acc3_a[j] = acc3_b[j] = 0.f;
      }
      int old = 0;
      const RopeKv rk{rk_f, rk_pos};
      if (publish_tile_rows<kGated, kF16, NT>(p, rt, u0, u1, gw, g, tok, lane, v, old, kRope ? &rk : nullptr)) {
        if (split_a < 0) {
          split_a = rt;
          old_a = old;
        } else {
          split_b = rt;
          old_b = old;
        }
      }
    }
  };

  for (int u = u0; u < u1; u += kDepth) {
#pragma unroll
    for (int dd = 0; dd < kDepth; ++dd) {
      if (u + dd < u1) {
        compute(sl[dd], u + dd);
        if (u + dd + kDepth < u1) load(sl[dd]);
      }
    }
  }
  const RopeKv rk{rk_f, rk_pos};
  if (split_a >= 0) finish_tile_rows<kGated, kF16, NT>(p, split_a, old_a, g, tok, lane, kRope ? &rk : nullptr);
  if (split_b >= 0) finish_tile_rows<kGated, kF16, NT>(p, split_b, old_b, g, tok, lane, kRope ? &rk : nullptr);
}

// ---------------------------------------------------------------------------
// block kernel: units of 16 rows x 64 codes, up to 4 column tiles of 8 rows
// ---------------------------------------------------------------------------

struct BlockSlot {
  uint2 wa, wb;
  float sa, sb;
  uint32_t qa, qb;
};

template <int NT, int P>
__global__ void __launch_bounds__(kThreads, 2) nf4_gemv_block_kernel(const GemvParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint8_t* lut = smem;
  const float* code2_s = reinterpret_cast<const float*>(smem + GEMV_LUT_BYTES);

  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * kWarps + (threadIdx.x >> 5);
  const bool active = gw < p.warps_total;
  const int u0 = active ? gw * p.uq + min(gw, p.ur) : 0;
  const int u1 = active ? u0 + p.uq + (gw < p.ur ? 1 : 0) : 0;
  const int g = lane >> 2, t = lane & 3;
  const int B = p.blocks_per_tile;  // 64-code units per row tile
  const int N = p.N, K = p.K, M = p.M;
  const int row_bytes = K >> 1;
  const uint32_t lane_base = (uint32_t)lane * 4u;
  const int nblk = K >> p.bs_shift;

  int lt = u0 / B, lk = u0 - (u0 / B) * B;
  int ct = lt, ck = lk;
  const uint8_t* pa = nullptr;
  const uint8_t* pb = nullptr;
  int ra = 0, rb = 0;
  auto set_rows = [&](int rt) {
    ra = min(rt * 16 + g, N - 1);
    rb = min(rt * 16 + g + 8, N - 1);
    pa = p.packed + (size_t)ra * row_bytes + t * 8;
    pb = p.packed + (size_t)rb * row_bytes + t * 8;
  };
  set_rows(lt);
  auto load = [&](int kb, BlockSlot& s) {
    s.wa = ld_stream_u2(pa + kb * 32);
    s.wb = ld_stream_u2(pb + kb * 32);
    const int ba = ra * nblk + ((kb * 64) >> p.bs_shift);
    const int bb = rb * nblk + ((kb * 64) >> p.bs_shift);
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

  BlockSlot ring[P];
#pragma unroll
  for (int i = 0; i < P; ++i)
    if (u0 + i < u1) {
      load(lk, ring[i]);
      if (++lk == B) { lk = 0; ++lt; set_rows(lt); }
    }
  build_tables(smem, p);
  __syncthreads();
  pdl_launch_dependents();
  if (!active) return;
  if (NF4B_GEMV_PREFETCH_EARLY) prefetch_next(p, gw, lane);

  pdl_wait();

  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;

  for (int base = u0; base < u1; base += P) {
#pragma unroll
    for (int i = 0; i < P; ++i) {
      const int u = base + i;
      if (u >= u1) break;
      const BlockSlot cur = ring[i];
      if (u + P < u1) {
        load(lk, ring[i]);
        if (++lk == B) { lk = 0; ++lt; set_rows(lt); }
      }
      const int rt = ct, kb = ck;
      if (++ck == B) { ck = 0; ++ct; }
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
        const int j0 = 2 * (s & 1);
        const uint32_t a0 = lut_lookup(lut, wa, lut_sel(j0), lane_base);
        const uint32_t a2 = lut_lookup(lut, wa, lut_sel(j0 + 1), lane_base);
        const uint32_t a1 = lut_lookup(lut, wb, lut_sel(j0), lane_base);
        const uint32_t a3 = lut_lookup(lut, wb, lut_sel(j0 + 1), lane_base);
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
        int rows[NT * 4], toks[NT * 4];
        float vals[NT * 4];
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            rows[j * 4 + e] = rt * 16 + g + ((e & 2) ? 8 : 0);
            toks[j * 4 + e] = j * 8 + 2 * t + (e & 1);
            vals[j * 4 + e] = acc[j][e];
          }
        finish_tile<NT * 4>(p, rt, u0, u1, gw, rows, toks, vals, lane);
#pragma unroll
        for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
      }
    }
  }
  if (!NF4B_GEMV_PREFETCH_EARLY) prefetch_next(p, gw, lane);
}

// ---------------------------------------------------------------------------
// GEMV chain: dependent decode GEMVs (rows <= 4, blocksize-64 weights with
// k_in % 256 == 0, x staged in shared memory) in ONE persistent launch
// ---------------------------------------------------------------------------
//
// Job j reads its x (and epilogue operand) only after every row tile of jobs
// 0..j-1 is stored, so x may be an earlier job's y. Units, runs, the unit
// loop and the split-tile protocol are the pair kernel's (256-code units,
// equal contiguous runs per warp, the last contributor to arrive reduces), so
// every job equals the separate call bit for bit. Each warp's TMA ring runs
// straight across job boundaries: the next job's first units are in flight
// while the current one finishes. A CTA counts itself into the job's
// completion count once all its warps are done with the job (reductions
// included); at the next boundary thread 0 waits (bounded) for the count to
// reach the grid size, then the CTA stages the job's code2 table(s) and x in
// one round trip - RMS-normalised first when the job asks for it, with the
// arithmetic of nf4b_rms_norm - behind a CTA barrier. The last CTA out
// re-zeroes the counts, so the workspace is left as it was found.

// The chain's view of a job as the pair kernel's split-tile helpers see it.
__device__ __forceinline__ void chain_as_params(const ChainJob& J, const ChainParams& cp, GemvParams& q) {
  q.N = J.N;
  q.M = cp.M;
  q.blocks_per_tile = J.B;
  q.uq = J.uq;
  q.ur = J.ur;
  q.partial = cp.partial;
  q.counters = cp.counters;
  q.y = J.y;
  q.operand = J.operand;
  q.epi = J.epi;
}

__global__ void __launch_bounds__(GEMV_PAIR_WARPS * 32, 1)
    nf4_gemv_chain_kernel(const __grid_constant__ ChainParams p) {
  constexpr int SU = 2;
  constexpr int R = GEMV_PAIR_STAGE_KB / SU;
  constexpr int WB = 1024 * SU, SB = 128 * SU;
  constexpr int kT = GEMV_PAIR_WARPS * 32;
  constexpr int XR = (GEMV_PAIR_X_MAX / 16 + kT - 1) / kT;  // x uint4s per thread at most
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ double red[GEMV_PAIR_WARPS];
  __shared__ int s_ok;
  const uint8_t* lut = smem;
  float* code2_s = reinterpret_cast<float*>(smem + GEMV_LUT_BYTES);
  float* code2_s3 = code2_s + 256;
  uint8_t* xs = smem + GEMV_PAIR_X_OFFSET;

  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int gw = blockIdx.x * GEMV_PAIR_WARPS + wib;
  const int g = lane >> 2, t = lane & 3;
  const int M = p.M, n_jobs = p.n_jobs;
  const uint32_t lane_base = (uint32_t)lane * 4u;
  int* done = p.counters + (GEMV_MAX_TILES - CHAIN_DONE_INTS);
  int* exit_ctr = done + (CHAIN_DONE_INTS - 1);

  const uint8_t* wring = smem + GEMV_PAIR_W_OFFSET + wib * (R * WB);
  const uint8_t* sring = smem + GEMV_PAIR_SC_OFFSET + wib * (R * SB);
  const uint32_t wring_s = smem_addr(wring), sring_s = smem_addr(sring);
  const uint32_t bar_s = smem_addr(smem + GEMV_PAIR_BAR_OFFSET + wib * (R * 8));
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < R; ++i) mbar_init1(bar_s + 8 * i);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (threadIdx.x == 0) s_ok = 1;
  __syncwarp();

  auto run_of = [&](int j, int& a, int& b) {
    const ChainJob& J = p.jobs[j];
    a = gw * J.uq + min(gw, J.ur);
    b = a + J.uq + (gw < J.ur ? 1 : 0);
  };

  // Load cursor: job lj, unit lu of this warp's run [lu, lend) in it, and the
  // unit's tile lt, half lh, k unit lk.
  int lj = -1, lu = 0, lend = 0, lt = 0, lh = 0, lk = 0;
  long long sbase = 0;  // first scale block of row g + 8t of tile lt
  auto load_rows = [&]() {
    const ChainJob& J = p.jobs[lj];
    sbase = (long long)min(lt * 16 + g + 8 * t, J.N - 1) * (J.K >> 6);
  };
  auto next_job = [&]() {
    while (++lj < n_jobs) {
      run_of(lj, lu, lend);
      if (lu < lend) {
        const ChainJob& J = p.jobs[lj];
        const int per_tile = J.gated ? 2 * J.B : J.B;
        lt = lu / per_tile;
        lk = lu - lt * per_tile;
        lh = 0;
        if (J.gated && lk >= J.B) {
          lh = 1;
          lk -= J.B;
        }
        load_rows();
        return;
      }
    }
  };
  next_job();
  auto step_load = [&]() {
    if (++lu == lend) {
      next_job();
      return;
    }
    const ChainJob& J = p.jobs[lj];
    if (++lk == J.B) {
      lk = 0;
      if (J.gated && lh == 0) {
        lh = 1;
      } else {
        lh = 0;
        ++lt;
      }
      load_rows();
    }
  };
  // The pair kernel's 256-code unit request: one TMA box, and per row one
  // aligned word of four scale codes plus the shared second-level scale (or
  // 16 bytes of fp32 scales).
  auto issue = [&](int st) {
    const ChainJob& J = p.jobs[lj];
    const bool h3 = J.gated && lh;
    if (lane == 0) {
      const uint32_t bar = bar_s + 8 * st;
      mbar_expect(bar, (uint32_t)WB);
      tma_box(wring_s + st * WB, h3 ? &J.wmap3 : &J.wmap, lk * 64 * SU, lt * 16, bar);
    }
    if (t < 2) {
      const uint32_t ds = sring_s + st * SB + (g + 8 * t) * (8 * SU);
      const long long be = sbase + lk * 4;  // four 64-blocks per unit, a multiple of 4
      const float* absmax = h3 ? J.absmax3 : J.absmax;
      if (J.nested) {
        cp_async_4(ds, (h3 ? J.a8_3 : J.a8) + be, 4u);
        cp_async_4(ds + 4, absmax + (be >> J.bs2_shift), 4u);
      } else {
        cp_async_16(ds, absmax + be);
      }
    }
  };

  int inflight = 0;  // unit copies requested and not yet consumed
#pragma unroll
  for (int i = 0; i < R - 1; ++i) {
    if (lj < n_jobs) {
      issue(i);
      step_load();
      ++inflight;
    }
    cp_async_commit();
  }
  build_pair_lut<kT>(smem);
  pdl_launch_dependents();
  pdl_wait();

  int st_use = 0, st_fill = R - 1;
  uint32_t phase = 0;
  for (int j = 0; j < n_jobs; ++j) {
    const ChainJob& J = p.jobs[j];
    GemvParams q;
    chain_as_params(J, p, q);
    // ---- job boundary: every CTA has stored its tiles of job j - 1
    if (j > 0 && threadIdx.x == 0) {
      const int need = (int)gridDim.x;
      if (!mbar_free_wait_count(done + (j - 1), need)) s_ok = 0;
    }
    __syncthreads();
    if (!s_ok) break;
    const int K = J.K;
    {
      // code2 and x in one round trip: every load issued before the stores
      const int n16 = (M * K) >> 3;
      const uint4* src = reinterpret_cast<const uint4*>(J.x);
      uint4 xv[XR];
#pragma unroll
      for (int r = 0; r < XR; ++r) {
        const int i = threadIdx.x + r * kT;
        if (i < n16) xv[r] = __ldcg(src + i);
      }
      float c2a = 0.f, c2b = 0.f;
      if (J.nested && threadIdx.x < 256) {
        c2a = __ldcg(J.code2 + threadIdx.x);
        if (J.gated) c2b = __ldcg(J.code2_3 + threadIdx.x);
      }
      uint4* dst = reinterpret_cast<uint4*>(xs);
#pragma unroll
      for (int r = 0; r < XR; ++r) {
        const int i = threadIdx.x + r * kT;
        if (i < n16) dst[i] = xv[r];
      }
      if (J.nested && threadIdx.x < 256) {
        code2_s[threadIdx.x] = c2a;
        if (J.gated) code2_s3[threadIdx.x] = c2b;
      }
    }
    __syncthreads();
    if (J.norm_w != nullptr) rms_normalise_staged<kT>(reinterpret_cast<uint16_t*>(xs), M, K, J.norm_w, J.norm_eps, red);

    // ---- this warp's units of job j (the pair kernel's unit loop)
    const int B = J.B, per_tile = J.gated ? 2 * B : B;
    int u0, u1;
    run_of(j, u0, u1);
    int ct = u0 / per_tile, ck = u0 - ct * per_tile, ch = 0;
    if (J.gated && ck >= B) {
      ch = 1;
      ck -= B;
    }
    const int xtok = g >> 1;
    const bool xlane = (xtok < M) && ((g & 1) == (t >> 1));
    const uint4* xrow = reinterpret_cast<const uint4*>(xs + (size_t)(xlane ? xtok : 0) * K * 2 + t * 64);
    float acc_a = 0.f, acc_b = 0.f, acc3_a = 0.f, acc3_b = 0.f;
    int split_a = -1, split_b = -1, old_a = 0, old_b = 0;
    for (int u = u0; u < u1; ++u) {
      __syncwarp();
      if (lj < n_jobs) {
        issue(st_fill);
        step_load();
        ++inflight;
      }
      cp_async_commit();
      st_fill = st_fill + 1 == R ? 0 : st_fill + 1;
      cp_async_wait<R - 1>();
      if (!mbar_wait_bounded(bar_s + 8 * st_use, (phase >> st_use) & 1u)) {
        drain_ring<R>(bar_s, st_use, inflight, phase);
        if (J.gated)
          abort_split_tiles<true>(q, ct, u0, u1, gw, g, t, lane, split_a, old_a, split_b, old_b);
        else
          abort_split_tiles<false>(q, ct, u0, u1, gw, g, t, lane, split_a, old_a, split_b, old_b);
        s_ok = 0;
        break;
      }
      --inflight;
      phase ^= 1u << st_use;
      __syncwarp();
      const uint8_t* wst = wring + st_use * WB;
      const uint8_t* sst = sring + st_use * SB;
      st_use = st_use + 1 == R ? 0 : st_use + 1;

      const int rt = ct, kb = ck, hh = ch;
      if (++ck == B) {
        ck = 0;
        if (J.gated && ch == 0) {
          ch = 1;
        } else {
          ch = 0;
          ++ct;
        }
      }
      const uint4 va = *reinterpret_cast<const uint4*>(sst + g * 16);
      const uint4 vb = *reinterpret_cast<const uint4*>(sst + (g + 8) * 16);
      const uint32_t sa[4] = {va.x, va.y, va.z, va.w}, sb[4] = {vb.x, vb.y, vb.z, vb.w};
      float ya = 0.f, yb = 0.f;
#pragma unroll
      for (int i = 0; i < SU; ++i) {
        const int kb2 = kb * SU + i;
        float se_a, so_a, se_b, so_b;
        if (J.nested) {
          const float* c2 = (J.gated && hh) ? code2_s3 : code2_s;
          const float off = (J.gated && hh) ? J.offset3 : J.offset;
          const uint32_t ea = (sa[0] >> (16 * i)) & 0xFFu, oa = (sa[0] >> (16 * i + 8)) & 0xFFu;
          const uint32_t eb = (sb[0] >> (16 * i)) & 0xFFu, ob = (sb[0] >> (16 * i + 8)) & 0xFFu;
          const float s2a = __uint_as_float(sa[1]), s2b = __uint_as_float(sb[1]);
          se_a = nested_scale(c2[ea], s2a, off);
          so_a = nested_scale(c2[oa], s2a, off);
          se_b = nested_scale(c2[eb], s2b, off);
          so_b = nested_scale(c2[ob], s2b, off);
        } else {
          se_a = __uint_as_float(sa[2 * i]); so_a = __uint_as_float(sa[2 * i + 1]);
          se_b = __uint_as_float(sb[2 * i]); so_b = __uint_as_float(sb[2 * i + 1]);
        }
        uint4 xq4[4];
        if (xlane) {
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) xq4[jj] = xrow[kb2 * 16 + jj];
        } else {
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) xq4[jj] = make_uint4(0, 0, 0, 0);
        }
        const uint4 wav = *reinterpret_cast<const uint4*>(wst + g * (64 * SU) + i * 64 + t * 16);
        const uint4 wbv = *reinterpret_cast<const uint4*>(wst + (g + 8) * (64 * SU) + i * 64 + t * 16);
        float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t wa[4] = {wav.x, wav.y, wav.z, wav.w};
        const uint32_t wb[4] = {wbv.x, wbv.y, wbv.z, wbv.w};
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const uint32_t w0 = wa[s >> 1], w1 = wb[s >> 1];
          const int j0 = 2 * (s & 1);
          const uint32_t a0 = lut_lookup(lut, w0, lut_sel(j0), lane_base);
          const uint32_t a2 = lut_lookup(lut, w0, lut_sel(j0 + 1), lane_base);
          const uint32_t a1 = lut_lookup(lut, w1, lut_sel(j0), lane_base);
          const uint32_t a3 = lut_lookup(lut, w1, lut_sel(j0 + 1), lane_base);
          const uint4& xq = xq4[s >> 1];
          const uint32_t b0 = (s & 1) ? xq.z : xq.x;
          const uint32_t b1 = (s & 1) ? xq.w : xq.y;
          if (s & 1)
            mma_bf16_16816(d1, a0, a1, a2, a3, b0, b1);
          else
            mma_bf16_16816(d0, a0, a1, a2, a3, b0, b1);
        }
        ya += fmaf(so_a, d0[1] + d1[1], (d0[0] + d1[0]) * se_a);
        yb += fmaf(so_b, d0[3] + d1[3], (d0[2] + d1[2]) * se_b);
      }
      if (J.gated && hh) {
        acc3_a += ya;
        acc3_b += yb;
      } else {
        acc_a += ya;
        acc_b += yb;
      }
      if ((kb == B - 1 && (!J.gated || hh == 1)) || u == u1 - 1) {
        const float v[2][2] = {{acc_a, acc_b}, {acc3_a, acc3_b}};
        int old = 0;
        const bool split = J.gated ? publish_pair_tile<true>(q, rt, u0, u1, gw, g, t, lane, v, old)
                                   : publish_pair_tile<false>(q, rt, u0, u1, gw, g, t, lane, v, old);
        if (split) {
          if (split_a < 0) {
            split_a = rt;
            old_a = old;
          } else {
            split_b = rt;
            old_b = old;
          }
        }
        acc_a = acc_b = acc3_a = acc3_b = 0.f;
      }
    }
    {  // after an abort too: the last contributor still re-zeroes each counter
      if (J.gated) {
        if (split_a >= 0) finish_split_tile<true>(q, split_a, old_a, g, t, lane);
        if (split_b >= 0) finish_split_tile<true>(q, split_b, old_b, g, t, lane);
      } else {
        if (split_a >= 0) finish_split_tile<false>(q, split_a, old_a, g, t, lane);
        if (split_b >= 0) finish_split_tile<false>(q, split_b, old_b, g, t, lane);
      }
    }
    // ---- this CTA is done with job j: count it in (release after the barrier)
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(done + j) : "memory");
    }
  }
  cp_async_wait<0>();
  // The last CTA out re-zeroes the completion counts for the next launch.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int old = atomicAdd(exit_ctr, 1);
    if (old == (int)gridDim.x - 1) {
      __threadfence();
      for (int j = 0; j < n_jobs; ++j) done[j] = 0;
      *exit_ctr = 0;
    }
  }
}

// ---------------------------------------------------------------------------
// Register-fed GEMV chain (rows <= 2): the register-fed pair kernel's unit
// body, runs and split tiles per job - so every job equals the separate call
// bit for bit - with each warp's three register slots running straight
// across job boundaries. At one activation row a warp owns 1-5 units of a
// decode projection, so most of the next job's weights are in flight while
// the CTA waits at the boundary. Job boundaries as in the chain above (one
// release add per CTA and job, a bounded wait for the grid, x and the code2
// copies staged in one round trip). A warp's unit count per job varies, so
// the slot of a job's first unit is only known at run time; the unit loop
// dispatches on it to one of three copies of the body, which keeps the slots
// in registers.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(GEMV_PAIR_WARPS * 32, 1)
    nf4_gemv_reg_chain_kernel(const __grid_constant__ ChainParams p) {
  constexpr int kT = GEMV_PAIR_WARPS * 32;
  constexpr int XR = (GEMV_PAIR_X_MAX / 16 + kT - 1) / kT;  // x uint4s per thread at most
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ double red[GEMV_PAIR_WARPS];
  __shared__ int s_ok;
  const uint8_t* lut = smem;
  uint8_t* xs = smem + GEMV_LUT_BYTES;

  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * GEMV_PAIR_WARPS + (threadIdx.x >> 5);
  const int g = lane >> 2, t = lane & 3;
  const int M = p.M, n_jobs = p.n_jobs;
  int* done = p.counters + (GEMV_MAX_TILES - CHAIN_DONE_INTS);
  int* exit_ctr = done + (CHAIN_DONE_INTS - 1);
  if (threadIdx.x == 0) s_ok = 1;

  auto run_of = [&](int j, int& a, int& b) {
    const ChainJob& J = p.jobs[j];
    a = gw * J.uq + min(gw, J.ur);
    b = a + J.uq + (gw < J.ur ? 1 : 0);
  };

  // Load cursor: job lj, unit lu of this warp's run [lu, lend) in it, and the
  // unit's tile lt, half lh, k unit lk; oa / ob = first 64-block of rows g, g + 8.
  int lj = -1, lu = 0, lend = 0, lt = 0, lh = 0, lk = 0, oa = 0, ob = 0;
  auto set_rows = [&]() {
    const ChainJob& J = p.jobs[lj];
    const int nblk = J.K >> 6;
    oa = min(lt * 16 + g, J.N - 1) * nblk;
    ob = min(lt * 16 + g + 8, J.N - 1) * nblk;
  };
  auto next_job = [&]() {
    while (++lj < n_jobs) {
      run_of(lj, lu, lend);
      if (lu < lend) {
        const ChainJob& J = p.jobs[lj];
        const int per_tile = J.gated ? 2 * J.B : J.B;
        lt = lu / per_tile;
        lk = lu - lt * per_tile;
        lh = 0;
        if (J.gated && lk >= J.B) {
          lh = 1;
          lk -= J.B;
        }
        set_rows();
        return;
      }
    }
  };
  next_job();
  auto load = [&](RegSlot& s) {
    if (lj >= n_jobs) return;
    const ChainJob& J = p.jobs[lj];
    const bool h3 = J.gated && lh;
    const uint8_t* pw = h3 ? J.packed3 : J.packed;
    const int ba = oa + lk * 4, bb = ob + lk * 4;
    ld_stream_u8(pw + (size_t)ba * 32 + t * 32, s.wa);
    ld_stream_u8(pw + (size_t)bb * 32 + t * 32, s.wb);
    const float* ps = h3 ? J.absmax3 : J.absmax;
    if (J.nested) {
      const uint8_t* pq = h3 ? J.a8_3 : J.a8;
      s.qa = __ldg(reinterpret_cast<const uint32_t*>(pq + ba));
      s.qb = __ldg(reinterpret_cast<const uint32_t*>(pq + bb));
      s.sa = __float_as_uint(__ldg(ps + (ba >> J.bs2_shift)));
      s.sb = __float_as_uint(__ldg(ps + (bb >> J.bs2_shift)));
    } else {
      const float2 fa = __ldg(reinterpret_cast<const float2*>(ps + ba + 2 * (t & 1)));
      const float2 fb = __ldg(reinterpret_cast<const float2*>(ps + bb + 2 * (t & 1)));
      s.qa = __float_as_uint(fa.x);
      s.sa = __float_as_uint(fa.y);
      s.qb = __float_as_uint(fb.x);
      s.sb = __float_as_uint(fb.y);
    }
    if (++lu == lend) {
      next_job();
      return;
    }
    if (++lk == J.B) {
      lk = 0;
      if (J.gated && lh == 0) {
        lh = 1;
      } else {
        lh = 0;
        ++lt;
        set_rows();
      }
    }
  };

  RegSlot sl[kRegDepth];
#pragma unroll
  for (int d = 0; d < kRegDepth; ++d)
    if (lj == 0) load(sl[d]);
  build_pair_lut_fast<kT>(smem);
  pdl_launch_dependents();
  pdl_wait();

  const uint32_t lane_base = (uint32_t)lane * 4u;
  const uint32_t c2_base = 128u + (uint32_t)(2 * g + (t & 1)) * 4u;
  const uint32_t qsel0 = 0x5504u | ((uint32_t)(2 * (t & 1)) << 4);
  const uint32_t qsel1 = 0x5504u | ((uint32_t)(2 * (t & 1) + 1) << 4);
  const int xtok = g >> 2;
  const bool xlane = (xtok < M) && ((g & 3) == t);
  const int tok = (t & 1) ? 7 : (t >> 1);
  for (int j = 0; j < n_jobs; ++j) {
    const ChainJob& J = p.jobs[j];
    // ---- job boundary: every CTA has stored its tiles of job j - 1
    if (j > 0 && threadIdx.x == 0) {
      if (!mbar_free_wait_count(done + (j - 1), (int)gridDim.x)) s_ok = 0;
    }
    __syncthreads();
    if (!s_ok) break;
    const int K = J.K, xrow = reg_x_row_bytes(K);
    {
      // x (padded) and the code2 copies in one round trip
      const int n16 = K >> 3, tot16 = M * n16;
      const uint4* src = reinterpret_cast<const uint4*>(J.x);
      float c2v[2048 / kT];
      if (J.nested) load_code2_copies<kT>(J.code2, J.gated ? J.code2_3 : nullptr, c2v);
      for (int r0 = 0; r0 < XR; r0 += 3) {  // three x loads in flight per thread (24 KB per CTA)
        uint4 xv[3];
#pragma unroll
        for (int r = 0; r < 3; ++r) {
          const int i = threadIdx.x + (r0 + r) * kT;
          if (i < tot16) xv[r] = __ldcg(src + i);
        }
#pragma unroll
        for (int r = 0; r < 3; ++r) {
          const int i = threadIdx.x + (r0 + r) * kT;
          if (i < tot16) {
            const int m = i / n16, cc = i - m * n16;
            *reinterpret_cast<uint4*>(xs + m * xrow + cc * 16 + (cc >> 3) * 16) = xv[r];
          }
        }
      }
      if (J.nested) store_code2_copies<kT>(smem, c2v);
    }
    __syncthreads();
    if (J.norm_w != nullptr)
      rms_normalise_staged<kT, true>(reinterpret_cast<uint16_t*>(xs), M, K, J.norm_w, J.norm_eps, red, xrow / 2);

    // ---- this warp's units of job j (the register-fed pair kernel's body),
    // compiled separately for gated and plain jobs (fewer live registers)
    int u0, u1;
    run_of(j, u0, u1);
    auto run_job = [&](auto gated_c) {
    constexpr bool gated = decltype(gated_c)::value;
    const int B = J.B, per_tile = gated ? 2 * B : B;
    const bool nested = J.nested;
    int ct = u0 / per_tile, ck = u0 - ct * per_tile, ch = 0;
    if (gated && ck >= B) {
      ch = 1;
      ck -= B;
    }
    const uint8_t* xb = xs + (xlane ? xtok : 0) * xrow + t * 144;
    float acc_a = 0.f, acc_b = 0.f, acc3_a = 0.f, acc3_b = 0.f;
    int split_a = -1, split_b = -1, old_a = 0, old_b = 0;
    auto compute = [&](const RegSlot& sv, int u) {
      const int rt = ct, kb = ck, hh = ch;
      if (++ck == B) {
        ck = 0;
        if (gated && ch == 0) {
          ch = 1;
        } else {
          ch = 0;
          ++ct;
        }
      }
      float s0a, s1a, s0b, s1b;
      if (nested) {
        const uint32_t cb = c2_base + ((gated && hh) ? 64u : 0u);
        const float off = (gated && hh) ? J.offset3 : J.offset;
        const float s2a = __uint_as_float(sv.sa), s2b = __uint_as_float(sv.sb);
        s0a = nested_scale(*reinterpret_cast<const float*>(lut + __byte_perm(sv.qa, cb, qsel0)), s2a, off);
        s1a = nested_scale(*reinterpret_cast<const float*>(lut + __byte_perm(sv.qa, cb, qsel1)), s2a, off);
        s0b = nested_scale(*reinterpret_cast<const float*>(lut + __byte_perm(sv.qb, cb, qsel0)), s2b, off);
        s1b = nested_scale(*reinterpret_cast<const float*>(lut + __byte_perm(sv.qb, cb, qsel1)), s2b, off);
      } else {
        s0a = __uint_as_float(sv.qa);
        s1a = __uint_as_float(sv.sa);
        s0b = __uint_as_float(sv.qb);
        s1b = __uint_as_float(sv.sb);
      }
      float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
      uint4 xv[4];
#pragma unroll
      for (int st = 0; st < 16; ++st) {
        if ((st & 7) == 0) {
          if (xlane) {
            const uint4* xr = reinterpret_cast<const uint4*>(xb + kb * 576 + (st >> 3) * 64);
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) xv[jj] = xr[jj];
          } else {
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) xv[jj] = make_uint4(0, 0, 0, 0);
          }
        }
        const uint32_t w0 = sv.wa[st >> 1], w1 = sv.wb[st >> 1];
        const int j0 = 2 * (st & 1);
        const uint32_t a0 = lut_lookup(lut, w0, lut_sel(j0), lane_base);
        const uint32_t a2 = lut_lookup(lut, w0, lut_sel(j0 + 1), lane_base);
        const uint32_t a1 = lut_lookup(lut, w1, lut_sel(j0), lane_base);
        const uint32_t a3 = lut_lookup(lut, w1, lut_sel(j0 + 1), lane_base);
        const uint4& xq = xv[(st >> 1) & 3];
        const uint32_t b0 = (st & 1) ? xq.z : xq.x;
        const uint32_t b1 = (st & 1) ? xq.w : xq.y;
        if (st & 1)
          mma_bf16_16816(d1, a0, a1, a2, a3, b0, b1);
        else
          mma_bf16_16816(d0, a0, a1, a2, a3, b0, b1);
      }
      const float ya = fmaf(s1a, d0[1] + d1[1], (d0[0] + d1[0]) * s0a);
      const float yb = fmaf(s1b, d0[3] + d1[3], (d0[2] + d1[2]) * s0b);
      if (gated && hh) {
        acc3_a += ya;
        acc3_b += yb;
      } else {
        acc_a += ya;
        acc_b += yb;
      }
      if ((kb == B - 1 && (!gated || hh == 1)) || u == u1 - 1) {
        acc_a += __shfl_xor_sync(0xffffffffu, acc_a, 1);
        acc_b += __shfl_xor_sync(0xffffffffu, acc_b, 1);
        acc3_a += __shfl_xor_sync(0xffffffffu, acc3_a, 1);
        acc3_b += __shfl_xor_sync(0xffffffffu, acc3_b, 1);
        const float v[2][2] = {{acc_a, acc_b}, {acc3_a, acc3_b}};
        int old = 0;
        GemvParams q;  // the split-tile helpers' view of the job, built where it is used
        chain_as_params(J, p, q);
        const bool split = gated ? publish_pair_tile<true>(q, rt, u0, u1, gw, g, tok, lane, v, old)
                                 : publish_pair_tile<false>(q, rt, u0, u1, gw, g, tok, lane, v, old);
        if (split) {
          if (split_a < 0) {
            split_a = rt;
            old_a = old;
          } else {
            split_b = rt;
            old_b = old;
          }
        }
        acc_a = acc_b = acc3_a = acc3_b = 0.f;
      }
    };
    // Slots 0..2 hold this warp's next units in order. Inside the job a slot
    // is refilled only with a unit of the same job; the next job's units are
    // requested after the split tiles are finished (below), so the finish
    // never holds three slots' registers, and still in flight during the
    // boundary wait.
    for (int u = u0; u < u1; u += kRegDepth) {
#pragma unroll
      for (int d = 0; d < kRegDepth; ++d) {
        if (u + d < u1) {
          compute(sl[d], u + d);
          if (u + d + kRegDepth < u1) load(sl[d]);
        }
      }
    }
    GemvParams q;
    chain_as_params(J, p, q);
    if (gated) {
      if (split_a >= 0) finish_split_tile<true>(q, split_a, old_a, g, tok, lane);
      if (split_b >= 0) finish_split_tile<true>(q, split_b, old_b, g, tok, lane);
    } else {
      if (split_a >= 0) finish_split_tile<false>(q, split_a, old_a, g, tok, lane);
      if (split_b >= 0) finish_split_tile<false>(q, split_b, old_b, g, tok, lane);
    }
    };
    if (J.gated)
      run_job(std::true_type{});
    else
      run_job(std::false_type{});
    // The next job's first units (up to three, into slots 0..2 in order),
    // requested now that every slot is free: they are in flight during the
    // boundary wait, and no slot is live while a split tile is finished.
#pragma unroll
    for (int d = 0; d < kRegDepth; ++d)
      if (lj == j + 1) load(sl[d]);
    // ---- this CTA is done with job j: count it in (release after the barrier)
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(done + j) : "memory");
    }
  }
  // The last CTA out re-zeroes the completion counts for the next launch.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int old = atomicAdd(exit_ctr, 1);
    if (old == (int)gridDim.x - 1) {
      __threadfence();
      for (int j = 0; j < n_jobs; ++j) done[j] = 0;
      *exit_ctr = 0;
    }
  }
}

template <typename Kernel>
cudaError_t launch_kernel(Kernel kernel, const GemvParams& p, int grid, cudaStream_t stream,
                          bool* configured, int smem = GEMV_SMEM_BYTES, int smem_max = GEMV_SMEM_BYTES,
                          int threads = kThreads) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

}  // namespace

static int g_sm_count[64];

int read_gemv_error(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemv_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_gemv_error, &zero, sizeof(int));
  }
  return v;
}

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



void gemv_plan(int N, int K, int M, int sm_count, bool pairs, GemvPlan* plan, bool gated, int su) {
  const long long tiles = (N + 15) / 16;
  const long long B = pairs ? K / (128 * su) : K / 64;
  const long long H = (pairs && gated) ? 2 : 1;  // halves per tile
  const long long U = tiles * B * H;
  const int wpc = pairs ? GEMV_PAIR_WARPS : kWarps;              // warps per CTA
  const long long ctas = (long long)sm_count * (pairs ? 1 : GEMV_CTAS_PER_SM);
  long long W = ctas * wpc;
  if (W > U) W = U;
  plan->tiles = tiles;
  plan->units = U;
  plan->blocks_per_tile = (int)B;
  plan->warps_total = (int)W;
  plan->grid = (int)((W + wpc - 1) / wpc);
  // Every warp owns at least floor(U / W) units, so a tile of B * H units
  // meets at most ceil(B * H / floor(U / W)) + 1 of them.
  const long long per = U / W;
  plan->slots = (int)((B * H + per - 1) / per + 1);
  plan->counter_bytes = GEMV_COUNTER_BYTES;
  plan->partial_bytes = (size_t)plan->slots * H * M * N * sizeof(float);
}

size_t chain_plan(ChainParams* p, int sm_count) {
  const long long W = (long long)sm_count * GEMV_PAIR_WARPS;
  p->warps_total = (int)W;
  size_t partial = 0;
  for (int i = 0; i < p->n_jobs; ++i) {
    ChainJob& J = p->jobs[i];
    const long long H = J.gated ? 2 : 1;
    J.B = J.K / 256;
    J.tiles = (J.N + 15) / 16;
    const long long U = (long long)J.tiles * J.B * H;
    J.uq = (int)(U / W);
    J.ur = (int)(U % W);
    // a tile of B * H units meets at most ceil(B * H / floor(U / W)) + 1 warps
    const long long per = J.uq > 0 ? J.uq : 1;
    const long long slots = (J.B * H + per - 1) / per + 1;
    const size_t bytes = (size_t)slots * H * p->M * J.N * sizeof(float);
    if (bytes > partial) partial = bytes;
  }
  return partial;
}

cudaError_t launch_gemv_chain(const ChainParams& p, cudaStream_t stream) {
  static bool configured[64] = {}, configured_reg[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !(p.reg ? configured_reg : configured)[dev]) {
    cudaError_t e = p.reg ? cudaFuncSetAttribute(nf4_gemv_reg_chain_kernel,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, GEMV_REG_SMEM_MAX)
                          : cudaFuncSetAttribute(nf4_gemv_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 GEMV_PAIR_SMEM_MAX);
    if (e != cudaSuccess) return e;
    (p.reg ? configured_reg : configured)[dev] = true;
  }
  int kmax = 0;
  for (int i = 0; i < p.n_jobs; ++i) kmax = p.jobs[i].K > kmax ? p.jobs[i].K : kmax;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(p.warps_total / GEMV_PAIR_WARPS));
  cfg.blockDim = dim3(GEMV_PAIR_WARPS * 32);
  cfg.dynamicSmemBytes = p.reg ? GEMV_LUT_BYTES + p.M * reg_x_row_bytes(kmax) : GEMV_PAIR_X_OFFSET + p.M * kmax * 2;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return p.reg ? cudaLaunchKernelEx(&cfg, nf4_gemv_reg_chain_kernel, p) : cudaLaunchKernelEx(&cfg, nf4_gemv_chain_kernel, p);
}

// The register-fed kernel's instantiation for (gated, nested, fp16, column tiles).
template <bool kGated, bool kNested, bool kF16, int NT>
cudaError_t launch_reg_nt(const GemvParams& p, int grid, cudaStream_t stream, int smem) {
  static bool configured[64] = {};
  return launch_kernel(nf4_gemv_reg_kernel<kGated, kNested, false, kF16, NT>, p, grid, stream, configured, smem,
                       GEMV_REG_SMEM_MAX, GEMV_PAIR_WARPS * 32);
}

template <bool kGated, bool kNested, bool kF16>
cudaError_t launch_reg_tiles(const GemvParams& p, int grid, cudaStream_t stream, int smem, int tiles) {
  if (tiles == 1) return launch_reg_nt<kGated, kNested, kF16, 1>(p, grid, stream, smem);
  if (tiles == 2) return launch_reg_nt<kGated, kNested, kF16, 2>(p, grid, stream, smem);
  return launch_reg_nt<kGated, kNested, kF16, 4>(p, grid, stream, smem);
}

template <bool kF16>
cudaError_t launch_reg_act(const GemvParams& p, int grid, cudaStream_t stream, int smem, int tiles) {
  if (p.gated)
    return p.nested ? launch_reg_tiles<true, true, kF16>(p, grid, stream, smem, tiles)
                    : launch_reg_tiles<true, false, kF16>(p, grid, stream, smem, tiles);
  return p.nested ? launch_reg_tiles<false, true, kF16>(p, grid, stream, smem, tiles)
                  : launch_reg_tiles<false, false, kF16>(p, grid, stream, smem, tiles);
}

cudaError_t launch_reg(const GemvParams& p, int grid, cudaStream_t stream, int smem, int tiles) {
  return p.f16 ? launch_reg_act<true>(p, grid, stream, smem, tiles) : launch_reg_act<false>(p, grid, stream, smem, tiles);
}

cudaError_t launch_gemv(const GemvParams& p, int grid, bool pairs, cudaStream_t stream) {
  static bool cfg_pair[64] = {}, cfg_gated[64] = {}, cfg_pair2[64] = {}, cfg_gated2[64] = {};
  static bool cfg1[64] = {}, cfg2[64] = {}, cfg4[64] = {};
  if (pairs && p.reg) {
    // column tiles: 1 for 1-2 rows, 2 for 3-4, 4 for 5-8
    const int smem = GEMV_LUT_BYTES + p.M * p.K * 2;
    const int nt = GEMV_PAIR_WARPS * 32;
    const int tiles = p.M <= 2 ? 1 : p.M <= 4 ? 2 : 4;
    if (p.rk_q != nullptr) {
      static bool cfg_rope[64] = {}, cfg_rope_plain[64] = {};
      if (p.f16 || tiles != 1) return cudaErrorInvalidValue;
      return p.nested ? launch_kernel(nf4_gemv_reg_kernel<false, true, true>, p, grid, stream, cfg_rope, smem,
                                      GEMV_REG_SMEM_MAX, nt)
                      : launch_kernel(nf4_gemv_reg_kernel<false, false, true>, p, grid, stream, cfg_rope_plain, smem,
                                      GEMV_REG_SMEM_MAX, nt);
    }
    return launch_reg(p, grid, stream, smem, tiles);
  }
  if (p.f16) return cudaErrorInvalidValue;  // fp16 is served by the register-fed kernel only
  if (pairs) {
    GemvParams q = p;
    const uint64_t rb = (uint64_t)p.K / 2;
    const uint32_t box = 64u * (uint32_t)p.su;
    if (!make_map_2d(&q.wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.packed, rb, (uint64_t)p.N, rb, box, 16,
                     CU_TENSOR_MAP_SWIZZLE_NONE) ||
        (p.gated && !make_map_2d(&q.wmap3, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.packed3, rb, (uint64_t)p.N, rb, box,
                                 16, CU_TENSOR_MAP_SWIZZLE_NONE)))
      return cudaErrorInvalidValue;
    const int smem = GEMV_PAIR_X_OFFSET + (p.x_staged ? p.M * p.K * 2 : 0);
    const int nt = GEMV_PAIR_WARPS * 32;
    if (p.su == 2)
      return p.gated ? launch_kernel(nf4_gemv_pair_kernel<true, 2>, q, grid, stream, cfg_gated2, smem,
                                     GEMV_PAIR_SMEM_MAX, nt)
                     : launch_kernel(nf4_gemv_pair_kernel<false, 2>, q, grid, stream, cfg_pair2, smem,
                                     GEMV_PAIR_SMEM_MAX, nt);
    return p.gated ? launch_kernel(nf4_gemv_pair_kernel<true, 1>, q, grid, stream, cfg_gated, smem,
                                   GEMV_PAIR_SMEM_MAX, nt)
                   : launch_kernel(nf4_gemv_pair_kernel<false, 1>, q, grid, stream, cfg_pair, smem,
                                   GEMV_PAIR_SMEM_MAX, nt);
  }
  if (p.M <= 8) return launch_kernel(nf4_gemv_block_kernel<1, 4>, p, grid, stream, cfg1);
  if (p.M <= 16) return launch_kernel(nf4_gemv_block_kernel<2, 2>, p, grid, stream, cfg2);
  return launch_kernel(nf4_gemv_block_kernel<4, 2>, p, grid, stream, cfg4);
}

}  // namespace nf4b
