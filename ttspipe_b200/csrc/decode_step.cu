// Persistent decode step: a sequence of dependent NF4 decode GEMVs (1 or 2
// activation rows) in ONE launch, with the weight stream running across the
// matmul boundaries.
//
// Replaces the per-matmul launches of one decode step - the reference issues
// nf4gemv.matmul for wqkv, wo (+residual), w1, w3 (silu gate) and w2
// (+residual) of every block in turn (app/engine/fusedlayer.py:212-269), and
// captures the step as a CUDA graph of those launches (app/engine/graphs.py).
// Every launch of a dependent matmul pays a serial handoff: the dependency
// release, x's round trip through L2 and the split tiles' reduction, while the
// weights - the bulk of the bytes - do not depend on x at all.
//
// Structure. One CTA of 16 warps per SM (a cooperative launch: all CTAs are
// resident, so they may wait on one another). Job j's units (16 weight rows x
// 256 codes, tile-major; a gated pair's tile is 16 rows of W1 then the same
// rows of W3) are split into equal contiguous ranges, one per CTA, and each
// CTA's range into 16 contiguous warp runs. The unit body is the register-fed
// GEMV's (gemv_unit.cuh): each lane loads its 64-blocks with 256-bit loads
// straight into registers, three units in flight per warp, pair-table
// dequantisation into mma.m16n8k16. Each warp requests its first unit of the
// next job as soon as its own run of the current job is computed, so it is
// in flight through the handoff; the other two once x is staged.
//
// Tiles. A tile inside one warp's run is finished by that warp. A tile shared
// by warps of one CTA is summed through shared memory in warp order. A tile
// shared by CTAs c_lo..c_hi is finished by c_hi: the others publish their
// CTA-level partial sums, c_hi adds them in CTA order to its own. All sums
// are in a fixed order, so results are deterministic (they differ from the
// separate nf4b_gemm call only in fp32 summation order).
//
// Handoff words. Finished outputs are published twice: into y (bf16, for the
// caller and for later jobs) and as 64-bit handoff words, each holding two
// adjacent bf16 outputs and a 32-bit flag = (launch epoch << 9) | (job + 1),
// written with one 64-bit store. The next job's CTAs poll the words they need
// directly: data and completion arrive in ONE L2 round trip, with no counter
// and no barrier. The epoch (kept in the workspace, advanced by the last CTA
// to leave each launch) makes every launch's flags new, so nothing is ever
// reset. Partial sums of split tiles travel the same way (fp32 + flag).
//
// Ordering. Everything a job reads that this launch produced comes from
// handoff words: x from the previous job's, an epilogue operand from the
// words of the previous job or the one before it (three regions in turn).
// A job whose x is the previous job's y stages x from them ("handoff
// boundary"; every CTA must finish at least one tile of that job, which the
// host checks). Any other boundary - x from elsewhere, an older job's output
// read from memory, a job too small - is a full barrier: each CTA fences
// (ordering all its earlier stores) and writes its arrival word, and every
// CTA polls all arrival words and fences before reading.
//
// Every wait is bounded (2 s of %globaltimer, or the test limit passed in
// the parameters); a CTA that gives up records it in the library's device
// error word (bit 3 of nf4b_device_error) and leaves, which makes the others
// give up in turn. No copy is in flight when a CTA leaves (the weights are
// loaded into registers), and the next launch's new epoch ignores whatever
// the abandoned launch wrote.

#include <type_traits>

#include "common.cuh"
#include "gemv_unit.cuh"
#include "kernels.cuh"

namespace nf4b {

namespace {

constexpr int kWarps = STEP_WARPS;
constexpr int kT = kWarps * 32;
// Shared memory: the pair table with the code2 copies, the warps' partial-sum
// slots [warp][slot][half][16 rows][2 activation rows], then x (padded).
constexpr int kSlotFloats = 2 * 2 * 16 * 2;
constexpr int kSlotBytes = kWarps * kSlotFloats * 4;
constexpr int kXOffset = GEMV_LUT_BYTES + kSlotBytes;
constexpr int kNormOffset = kXOffset + 2 * reg_x_row_bytes(STEP_MAX_K);
constexpr int kSmemBytes = kNormOffset + 2 * STEP_MAX_K;
static_assert(kNormOffset % 16 == 0 && kSmemBytes <= 227 * 1024, "decode step shared memory layout");

__device__ int g_step_error = 0;  // bit 3 of nf4b_device_error: a handoff or barrier wait gave up

__device__ __forceinline__ unsigned long long step_timer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void word_store(uint64_t* p, uint32_t data, uint32_t flag) {
  const uint64_t v = ((uint64_t)flag << 32) | data;
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t word_load(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// Poll the word at p until its flag is `flag` (bounded by `limit` ns); its
// data, or 0 after recording the timeout and clearing `ok` (a thread whose
// `ok` is already clear does not wait at all).
__device__ __forceinline__ uint32_t word_wait(const uint64_t* p, uint64_t first, uint32_t flag,
                                              unsigned long long limit, bool& ok) {
  uint64_t v = first;
  if ((uint32_t)(v >> 32) == flag) return (uint32_t)v;
  if (!ok) return 0u;  // this thread gave up before: do not wait again
  const unsigned long long start = step_timer();
  for (uint32_t i = 1;; ++i) {
    v = word_load(p);
    if ((uint32_t)(v >> 32) == flag) return (uint32_t)v;
    if ((i & 31u) == 0u && step_timer() - start > limit) {
      atomicOr(&g_step_error, 8);
      ok = false;
      return 0u;
    }
  }
}

// Wait for a batch of words at once: w[r] (r < NB, bit r of `live`) holds a
// first read of the word at addr(r); every word whose flag is not yet `flag`
// is read again, all of them together, until none is stale - one L2 round
// trip per round however many are stale (bounded by `limit` ns; after a
// timeout the stale words read 0 and `ok` is cleared).
template <int NB, class Addr>
__device__ __forceinline__ void words_wait(uint64_t (&w)[NB], uint32_t live, Addr addr, uint32_t flag,
                                           unsigned long long limit, bool& ok) {
  uint32_t pend = 0;
#pragma unroll
  for (int r = 0; r < NB; ++r)
    if (((live >> r) & 1u) && (uint32_t)(w[r] >> 32) != flag) pend |= 1u << r;
  if (pend == 0u) return;
  const unsigned long long start = ok ? step_timer() : 0ull;
  for (uint32_t i = 0; pend != 0u; ++i) {
    if (!ok || ((i & 15u) == 15u && step_timer() - start > limit)) {
      if (ok) atomicOr(&g_step_error, 8);
      ok = false;
#pragma unroll
      for (int r = 0; r < NB; ++r)
        if ((pend >> r) & 1u) w[r] = 0ull;
      return;
    }
#pragma unroll
    for (int r = 0; r < NB; ++r)
      if ((pend >> r) & 1u) w[r] = word_load(addr(r));
#pragma unroll
    for (int r = 0; r < NB; ++r)
      if (((pend >> r) & 1u) && (uint32_t)(w[r] >> 32) == flag) pend &= ~(1u << r);
  }
}

// The small tables job j reads at its start - the fused norm's weight and the
// code2 table(s) - streamed into L2 while the job before it runs, so staging
// does not wait on HBM for them (one bulk prefetch each; the host checks
// their 16-byte alignment and sizes).
__device__ __forceinline__ void prefetch_tables(const StepJob& J) {
  if (J.norm_w != nullptr)
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(J.norm_w), "r"((uint32_t)J.K * 2u) : "memory");
  if (J.nested) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], 1024;" ::"l"(J.code2) : "memory");
    if (J.gated) asm volatile("cp.async.bulk.prefetch.L2.global [%0], 1024;" ::"l"(J.code2_3) : "memory");
  }
}

__device__ __forceinline__ uint32_t job_flag(uint32_t epoch, int j) { return (epoch << 9) | (uint32_t)(j + 1); }

// Unit range of CTA c in a job of U units over G CTAs, and the CTA owning unit u.
__device__ __forceinline__ void cta_range(long long U, int G, int c, int& a, int& b) {
  a = (int)(U * c / G);
  b = (int)(U * (c + 1) / G);
}
__device__ __forceinline__ int cta_of(long long u, long long U, int G) { return (int)(((u + 1) * G - 1) / U); }

// The handoff words of job j: finals [tiles * 8 pairs][M], then partials
// [tiles][smax - 1][H][16 rows][M]. Three regions in turn: job j's words stay
// until job j + 3 writes its own, so a job can read its operand from the
// words of the job two before it.
__device__ __forceinline__ uint64_t* region_of(const StepParams& p, int j) { return p.ll[j % 3]; }

__global__ void __launch_bounds__(kT, 1) nf4_decode_step_kernel(const __grid_constant__ StepParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ double norm_red[2 * kWarps];
  __shared__ uint32_t s_epoch;
  __shared__ int s_last;
  const uint8_t* lut = smem;
  float* sp = reinterpret_cast<float*>(smem + GEMV_LUT_BYTES);
  uint8_t* xs = smem + kXOffset;
  uint16_t* wn = reinterpret_cast<uint16_t*>(smem + kNormOffset);  // the fused norm's weight

  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int c = blockIdx.x, G = gridDim.x;
  const int M = p.M, n_jobs = p.n_jobs;
  const unsigned long long limit = p.wait_ns;

  bool alive = true;  // this thread saw no wait give up (decided CTA-wide by __syncthreads_or)
  if (threadIdx.x == 0) {
    uint32_t e;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(e) : "l"(p.epoch) : "memory");
    s_epoch = e;
  }

  // This warp's run of job j: [a, b) within the CTA's range.
  auto run_of = [&](int j, int& a, int& b) {
    int ca, cb;
    cta_range(p.jobs[j].units, G, c, ca, cb);
    const int n = cb - ca;
    a = ca + n * wib / kWarps;
    b = ca + n * (wib + 1) / kWarps;
  };

  // Load cursor: job lj, unit lu of this warp's run [lu, lend) in it, and the
  // unit's tile lt, half lh, k unit lk; oa / ob = first 64-block of rows g, g + 8.
  int lj = -1, lu = 0, lend = 0, lt = 0, lh = 0, lk = 0, oa = 0, ob = 0;
  auto set_rows = [&]() {
    const StepJob& J = p.jobs[lj];
    const int nblk = J.K >> 6;
    oa = (lt * 16 + g) * nblk;
    ob = (lt * 16 + g + 8) * nblk;
  };
  auto next_job = [&]() {
    while (++lj < n_jobs) {
      run_of(lj, lu, lend);
      if (lu < lend) {
        const StepJob& J = p.jobs[lj];
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
    const StepJob& J = p.jobs[lj];
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
  int ahead = 0;  // units of the coming job already loaded (into slot 0) across its handoff
  if (threadIdx.x == 0) prefetch_tables(p.jobs[0]);
  build_pair_lut_fast<kT>(smem);
  __syncthreads();
  const uint32_t epoch = s_epoch;

  const uint32_t lane_base = (uint32_t)lane * 4u;
  const uint32_t c2_base = 128u + (uint32_t)(2 * g + (t & 1)) * 4u;
  const uint32_t qsel0 = 0x5504u | ((uint32_t)(2 * (t & 1)) << 4);
  const uint32_t qsel1 = 0x5504u | ((uint32_t)(2 * (t & 1) + 1) << 4);
  const int xtok = g >> 2;
  const bool xlane = (xtok < M) && ((g & 3) == t);
  const int tok = (t & 1) ? 7 : (t >> 1);  // the activation row this lane finishes (7: none)

  for (int j = 0; j < n_jobs; ++j) {
    const StepJob& J = p.jobs[j];
    // ---- boundary: job j - 1 is complete where this job reads it
    if (j > 0) {
      const StepJob& P = p.jobs[j - 1];
      if (P.barrier || j == p.stall_job) {
        if (threadIdx.x < G) {
          // the test hook expects a flag no launch writes (bit 8 set), so the wait runs out
          const uint32_t want = job_flag(epoch, j - 1) | (j == p.stall_job ? 0x100u : 0u);
          const uint64_t* w = p.arrive + (size_t)((j - 1) & 1) * G + threadIdx.x;
          (void)word_wait(w, word_load(w), want, limit, alive);
          fence_gpu();
        }
        if (__syncthreads_or(!alive)) break;
      }
    }
    const int K = J.K, xrow = reg_x_row_bytes(K);
    const bool normed = J.norm_w != nullptr;
    {
      // code2 copies of this job's weight(s), the norm weight, and x - from
      // the previous job's handoff words or from memory - with the fp64 sum of
      // squares of every row the fused RMSNorm needs (nf4b_rms_norm's
      // arithmetic: each square of a bf16 value is exact in fp64)
      float c2v[2048 / kT];
      if (J.nested) load_code2_copies<kT>(J.code2, J.gated ? J.code2_3 : nullptr, c2v);
      double ss0 = 0.0, ss1 = 0.0;
      auto sq2 = [&](int m, uint32_t v) {
        const double a = bf2f((bf16_t)(v & 0xFFFFu)), b = bf2f((bf16_t)(v >> 16));
        if (m == 0) ss0 += a * a + b * b; else ss1 += a * a + b * b;
      };
      // the norm weight (<= 3 x 16 bytes per thread) is requested before any
      // wait and stored once x is in
      uint4 nv[(STEP_MAX_K / 8 + kT - 1) / kT];
      if (normed) {
        const uint4* nsrc = reinterpret_cast<const uint4*>(J.norm_w);
#pragma unroll
        for (int r = 0; r < (STEP_MAX_K / 8 + kT - 1) / kT; ++r) {
          const int i = threadIdx.x + r * kT;
          if (i < (K >> 3)) nv[r] = __ldg(nsrc + i);
        }
      }
      if (J.x_ll) {
        const uint64_t* fw = region_of(p, j - 1);
        const uint32_t want = job_flag(epoch, j - 1);
        const int total = (K >> 1) * M;  // words: one per pair of x values and activation row
        for (int base = 0; base < total; base += 8 * kT) {
          uint64_t w[8];
          uint32_t live = 0;
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            const int idx = base + threadIdx.x + r * kT;
            w[r] = 0ull;
            if (idx < total) {
              w[r] = word_load(fw + idx);
              live |= 1u << r;
            }
          }
          words_wait(w, live, [&](int r) { return fw + base + threadIdx.x + r * kT; }, want, limit, alive);
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            const int idx = base + threadIdx.x + r * kT;
            if (idx < total) {
              const int m = idx % M, e = (idx / M) * 2;
              *reinterpret_cast<uint32_t*>(xs + m * xrow + 2 * e + (e >> 6) * 16) = (uint32_t)w[r];
              if (normed) sq2(m, (uint32_t)w[r]);
            }
          }
        }
      } else {
        const int n16 = K >> 3, tot16 = M * n16;
        const uint4* src = reinterpret_cast<const uint4*>(J.x);
        for (int i0 = 0; i0 < tot16; i0 += 4 * kT) {
          uint4 xv[4];
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const int i = i0 + threadIdx.x + r * kT;
            if (i < tot16) xv[r] = __ldcg(src + i);
          }
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const int i = i0 + threadIdx.x + r * kT;
            if (i < tot16) {
              const int m = i / n16, cc = i - m * n16;
              *reinterpret_cast<uint4*>(xs + m * xrow + cc * 16 + (cc >> 3) * 16) = xv[r];
              if (normed) {
                sq2(m, xv[r].x);
                sq2(m, xv[r].y);
                sq2(m, xv[r].z);
                sq2(m, xv[r].w);
              }
            }
          }
        }
      }
      if (J.nested) store_code2_copies<kT>(smem, c2v);
      if (normed) {
#pragma unroll
        for (int r = 0; r < (STEP_MAX_K / 8 + kT - 1) / kT; ++r) {
          const int i = threadIdx.x + r * kT;
          if (i < (K >> 3)) reinterpret_cast<uint4*>(wn)[i] = nv[r];
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
          ss0 += __shfl_xor_sync(0xffffffffu, ss0, off);
          ss1 += __shfl_xor_sync(0xffffffffu, ss1, off);
        }
        if (lane == 0) {
          norm_red[wib] = ss0;
          norm_red[kWarps + wib] = ss1;
        }
      }
    }
    if (__syncthreads_or(!alive)) break;
    if (threadIdx.x == 0 && j + 1 < n_jobs) prefetch_tables(p.jobs[j + 1]);
    // This job's first units into registers (the first may already be in
    // flight since the end of the previous job; they arrive while x is
    // normalised).
#pragma unroll
    for (int d = 0; d < kRegDepth; ++d)
      if (d >= ahead && lj == j) load(sl[d]);
    if (normed) {
      // y = bf16(bf16(x * r) * w), r = 1 / sqrt(fp32(ss / K) + eps), in place
      for (int m = 0; m < M; ++m) {
        double tot = 0.0;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) tot += norm_red[m * kWarps + w];
        const float r = rsqrt_exact(tot, K, J.norm_eps);
        uint16_t* xr = reinterpret_cast<uint16_t*>(xs + m * xrow);
        for (int i = threadIdx.x; i < (K >> 1); i += kT) {
          const int e = 2 * i;
          uint32_t* px = reinterpret_cast<uint32_t*>(xr + e + ((e >> 6) << 3));
          const uint32_t xv = *px, wv = *reinterpret_cast<const uint32_t*>(wn + e);
          const float n0 = round_bf(__fmul_rn(bf2f((bf16_t)(xv & 0xFFFFu)), r));
          const float n1 = round_bf(__fmul_rn(bf2f((bf16_t)(xv >> 16)), r));
          *px = (uint32_t)f2bf(__fmul_rn(n0, bf2f((bf16_t)(wv & 0xFFFFu)))) |
                ((uint32_t)f2bf(__fmul_rn(n1, bf2f((bf16_t)(wv >> 16)))) << 16);
        }
      }
      __syncthreads();
    }

    // ---- this warp's units of job j
    int ca, cb, u0, u1;
    cta_range(J.units, G, c, ca, cb);
    run_of(j, u0, u1);
    const uint32_t flag = job_flag(epoch, j);
    uint64_t* region = region_of(p, j);
    const int N = J.N;
    const int smax1 = J.smax - 1;
    uint64_t* partials = region + (size_t)J.tiles * 8 * M;
    const uint64_t* op_final = J.op_ll ? region_of(p, j - J.op_ll) : nullptr;
    const uint32_t op_flag = J.op_ll ? job_flag(epoch, j - J.op_ll) : 0u;

    // Store tile rt's outputs (fp32 sums v[half][row g / g + 8] of activation
    // row tok): the epilogue or the gate, y, and the handoff words (two
    // adjacent rows per word). Called by whole warps.
    auto final_store = [&](int rt, const float (&v)[2][2], bool& okf) {
      const int ra = rt * 16 + g, rb = ra + 8;
      uint32_t ya = 0u, yb = 0u;
      if (tok < M) {
        if (J.gated) {
          ya = gate_bf16(v[0][0], v[1][0]);
          yb = gate_bf16(v[0][1], v[1][1]);
        } else {
          float opa = 0.f, opb = 0.f;
          if (J.epi != NF4B_EPI_NONE) {
            if (J.op_ll) {  // job j - op_ll's y: read from its handoff words
              const uint64_t* wa = op_final + (size_t)(ra >> 1) * M + tok;
              const uint64_t* wb = op_final + (size_t)(rb >> 1) * M + tok;
              uint64_t pw[2] = {word_load(wa), word_load(wb)};
              words_wait(pw, 3u, [&](int r) { return r ? wb : wa; }, op_flag, limit, okf);
              const uint32_t pa = (uint32_t)pw[0], pb = (uint32_t)pw[1];
              opa = bf2f((bf16_t)((ra & 1) ? pa >> 16 : pa & 0xFFFFu));
              opb = bf2f((bf16_t)((rb & 1) ? pb >> 16 : pb & 0xFFFFu));
            } else {
              opa = bf2f(__ldcg(J.operand + (size_t)tok * N + ra));
              opb = bf2f(__ldcg(J.operand + (size_t)tok * N + rb));
            }
          }
          ya = epilogue_value(v[0][0], J.epi, opa);
          yb = epilogue_value(v[0][1], J.epi, opb);
        }
        J.y[(size_t)tok * N + ra] = (bf16_t)ya;
        J.y[(size_t)tok * N + rb] = (bf16_t)yb;
      }
      // rows g + 1 (lane + 4) pair up with rows g for even g
      const uint32_t na = __shfl_down_sync(0xffffffffu, ya, 4);
      const uint32_t nb = __shfl_down_sync(0xffffffffu, yb, 4);
      if (tok < M && (g & 1) == 0) {
        word_store(region + ((size_t)rt * 8 + (g >> 1)) * M + tok, ya | (na << 16), flag);
        word_store(region + ((size_t)rt * 8 + 4 + (g >> 1)) * M + tok, yb | (nb << 16), flag);
      }
    };

    auto run_job = [&](auto gated_c) {
      constexpr bool gated = decltype(gated_c)::value;
      const int B = J.B, P = gated ? 2 * B : B;
      const bool nested = J.nested;
      const int tile_first = u0 / P, tile_last = (u1 - 1) / P;
      int ct = u0 / P, ck = u0 - ct * P, ch = 0;
      if (gated && ck >= B) {
        ch = 1;
        ck -= B;
      }
      const uint8_t* xb = xs + (xlane ? xtok : 0) * xrow + t * 144;
      float acc_a = 0.f, acc_b = 0.f, acc3_a = 0.f, acc3_b = 0.f;
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
          const uint32_t cbs = c2_base + ((gated && hh) ? 64u : 0u);
          const float off = (gated && hh) ? J.offset3 : J.offset;
          const float s2a = __uint_as_float(sv.sa), s2b = __uint_as_float(sv.sb);
          s0a = nested_scale(*reinterpret_cast<const float*>(lut + __byte_perm(sv.qa, cbs, qsel0)), s2a, off);
          s1a = nested_scale(*reinterpret_cast<const float*>(lut + __byte_perm(sv.qa, cbs, qsel1)), s2a, off);
          s0b = nested_scale(*reinterpret_cast<const float*>(lut + __byte_perm(sv.qb, cbs, qsel0)), s2b, off);
          s1b = nested_scale(*reinterpret_cast<const float*>(lut + __byte_perm(sv.qb, cbs, qsel1)), s2b, off);
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
          if (gated) {
            acc3_a += __shfl_xor_sync(0xffffffffu, acc3_a, 1);
            acc3_b += __shfl_xor_sync(0xffffffffu, acc3_b, 1);
          }
          const long long t0 = (long long)rt * P;
          if (t0 >= u0 && t0 + P <= u1) {  // the whole tile is this warp's
            const float v[2][2] = {{acc_a, acc_b}, {acc3_a, acc3_b}};
            final_store(rt, v, alive);
          } else if (tok < M) {  // a share of a tile: into this warp's slot
            float* s = sp + (size_t)(wib * 2 + (rt == tile_first ? 0 : 1)) * (2 * 16 * 2);
            s[(0 * 16 + g) * 2 + tok] = acc_a;
            s[(0 * 16 + g + 8) * 2 + tok] = acc_b;
            if (gated) {
              s[(1 * 16 + g) * 2 + tok] = acc3_a;
              s[(1 * 16 + g + 8) * 2 + tok] = acc3_b;
            }
          }
          acc_a = acc_b = acc3_a = acc3_b = 0.f;
        }
      };
      for (int u = u0; u < u1; u += kRegDepth) {
#pragma unroll
        for (int d = 0; d < kRegDepth; ++d) {
          if (u + d < u1) {
            compute(sl[d], u + d);
            if (u + d + kRegDepth < u1) load(sl[d]);
          }
        }
      }
      (void)tile_last;
    };
    if (u0 < u1) {
      if (J.gated)
        run_job(std::true_type{});
      else
        run_job(std::false_type{});
    }
    // The next job's first unit, in flight through the handoff (one per warp:
    // more would delay the handoff's own loads).
    ahead = 0;
    if (lj == j + 1) {
      load(sl[0]);
      ahead = 1;
    }
    __syncthreads();  // every warp's slot shares are in shared memory

    // ---- tiles shared by warps or CTAs: each is finished by the first warp
    // of this CTA that holds a share of it
    if (u0 < u1) {
      const int H = J.gated ? 2 : 1, P = J.gated ? 2 * J.B : J.B;
      const long long U = J.units;
      const int tf = u0 / P, tl = (u1 - 1) / P;
      for (int pass = 0; pass < 2; ++pass) {
        const int rt = pass == 0 ? tf : tl;
        if (pass == 1 && tl == tf) break;
        const long long t0 = (long long)rt * P, t1 = t0 + P;  // the tile's units [t0, t1)
        if (t0 >= u0 && t1 <= u1) continue;                    // finished in the unit loop
        const long long first = t0 > ca ? t0 : ca;              // the CTA's first unit of the tile
        if (first < u0 || first >= u1) continue;               // another warp finishes it
        const long long last = (t1 < cb ? t1 : cb) - 1;
        // the warps holding shares: runs containing first .. last
        const int n = cb - ca;
        const int w_lo = (int)(((first - ca + 1) * kWarps - 1) / n);
        const int w_hi = (int)(((last - ca + 1) * kWarps - 1) / n);
        float v[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
        if (tok < M) {
          for (int w = w_lo; w <= w_hi; ++w) {
            const int wa = ca + n * w / kWarps, wb = ca + n * (w + 1) / kWarps;
            if (wa == wb) continue;  // an empty run (fewer units than warps) holds no share
            const int slot = (rt == wa / P) ? 0 : 1;
            const float* s = sp + (size_t)(w * 2 + slot) * (2 * 16 * 2);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              if (h < H) {
                v[h][0] += s[(h * 16 + g) * 2 + tok];
                v[h][1] += s[(h * 16 + g + 8) * 2 + tok];
              }
            }
          }
        }
        if (t0 >= ca && t1 <= cb) {  // the whole tile is this CTA's
          final_store(rt, v, alive);
          continue;
        }
        const int c_lo = cta_of(t0, U, G), c_hi = cta_of(t1 - 1, U, G);
        if (c < c_hi) {  // publish this CTA's share for c_hi
          if (tok < M) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              if (h < H) {
                uint64_t* pw = partials + ((((size_t)rt * smax1 + (c - c_lo)) * H + h) * 16) * M + tok;
                word_store(pw + (size_t)g * M, __float_as_uint(v[h][0]), flag);
                word_store(pw + (size_t)(g + 8) * M, __float_as_uint(v[h][1]), flag);
              }
            }
          }
        } else {  // c_hi: add the other CTAs' shares in CTA order, then this one's
          float tot[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
          if (tok < M) {
            for (int s = 0; s < c_hi - c_lo; ++s) {
              // a CTA between the tile's first and last owner with an empty
              // range (a job of fewer units than CTAs) holds no share
              int sa_, sb_;
              cta_range(U, G, c_lo + s, sa_, sb_);
              if (sa_ == sb_) continue;
              const uint64_t* pw = partials + (((size_t)rt * smax1 + s) * H) * 16 * M + tok;
              // word r: half r >> 1, row g (r even) or g + 8 (r odd)
              auto at = [&](int r) { return pw + ((size_t)(r >> 1) * 16 + g + 8 * (r & 1)) * M; };
              uint64_t q[4];
              const uint32_t live = H == 2 ? 15u : 3u;
#pragma unroll
              for (int r = 0; r < 4; ++r) q[r] = ((live >> r) & 1u) ? word_load(at(r)) : 0ull;
              words_wait(q, live, at, flag, limit, alive);
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                if (h < H) {
                  tot[h][0] += __uint_as_float((uint32_t)q[2 * h]);
                  tot[h][1] += __uint_as_float((uint32_t)q[2 * h + 1]);
                }
              }
            }
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            tot[h][0] += v[h][0];
            tot[h][1] += v[h][1];
          }
          final_store(rt, tot, alive);
        }
      }
    }
    if (J.barrier) {
      // a full barrier follows: count this CTA in once all its stores are out
      __syncthreads();
      if (threadIdx.x == 0) {
        fence_gpu();
        word_store(p.arrive + (size_t)(j & 1) * G + c, 0u, flag);
      }
    }
  }

  // ---- leave: the last CTA out advances the epoch (a new flag space for the
  // next launch; at a wrap of its 23 bits the handoff words are cleared first)
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_gpu();
    const int old = atomicAdd(p.exit_ctr, 1);
    s_last = old == G - 1;
  }
  __syncthreads();
  if (s_last) {
    const uint32_t next = (epoch + 1u) & 0x7FFFFFu;
    if (next == 0u) {
      for (long long i = threadIdx.x; i < p.ll_words; i += kT) {
        p.ll[0][i] = 0ull;
        p.ll[1][i] = 0ull;
        p.ll[2][i] = 0ull;
      }
      for (int i = threadIdx.x; i < 2 * G; i += kT) p.arrive[i] = 0ull;
      __syncthreads();
    }
    if (threadIdx.x == 0) {
      fence_gpu();
      *p.exit_ctr = 0;
      asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p.epoch), "r"(next) : "memory");
    }
  }
}

}  // namespace

size_t step_plan(StepParams* p, int sm_count) {
  const int G = sm_count;
  p->grid = G;
  long long words = 0;
  for (int i = 0; i < p->n_jobs; ++i) {
    StepJob& J = p->jobs[i];
    const long long H = J.gated ? 2 : 1;
    J.B = J.K / 256;
    J.tiles = (J.N + 15) / 16;
    const long long P = (long long)J.B * H;
    const long long U = (long long)J.tiles * P;
    J.units = (int)U;
    // the most CTAs one tile meets
    int smax = 1;
    for (long long tl = 0; tl < J.tiles; ++tl) {
      const long long c_lo = ((tl * P + 1) * G - 1) / U, c_hi = (((tl + 1) * P) * G - 1) / U;
      if (c_hi - c_lo + 1 > smax) smax = (int)(c_hi - c_lo + 1);
    }
    J.smax = smax;
    const long long w = (long long)J.tiles * 8 * p->M + (long long)J.tiles * (smax - 1) * H * 16 * p->M;
    if (w > words) words = w;
  }
  // Which earlier job produced a pointer (-1: none of them).
  auto producer = [&](const void* ptr, int before) {
    for (int k = before - 1; k >= 0; --k)
      if (ptr == p->jobs[k].y) return k;
    return -1;
  };
  for (int i = 0; i < p->n_jobs; ++i) {
    StepJob& J = p->jobs[i];
    J.x_ll = 0;
    J.op_ll = 0;
    J.barrier = 0;
  }
  for (int i = 1; i < p->n_jobs; ++i) {
    StepJob& J = p->jobs[i];
    StepJob& pv = p->jobs[i - 1];
    // a handoff boundary needs every CTA to finish a tile of the previous
    // job: each CTA's range (>= floor(U / G) units) then holds a tile's last unit
    const bool covers = (long long)pv.units / G >= (long long)pv.B * (pv.gated ? 2 : 1);
    const int xp = producer(J.x, i);
    bool barrier = false;
    if (xp == i - 1 && covers) J.x_ll = 1;
    else barrier = true;  // x from memory: written before this launch, or ordered by the barrier
    if (J.operand != nullptr) {
      const int op = producer(J.operand, i);
      if (op >= 0 && i - op <= 2) J.op_ll = i - op;
      else if (op >= 0) barrier = true;
    }
    pv.barrier = barrier ? 1 : 0;
  }
  p->ll_words = words;
  return (size_t)STEP_CONTROL_BYTES + (size_t)2 * G * 8 + (size_t)3 * words * 8;
}

cudaError_t launch_decode_step(StepParams& p, void* workspace, cudaStream_t stream) {
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int smem = kSmemBytes;
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(nf4_decode_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.epoch = reinterpret_cast<unsigned*>(ws);
  p.exit_ctr = reinterpret_cast<int*>(ws + 4);
  p.arrive = reinterpret_cast<uint64_t*>(ws + STEP_CONTROL_BYTES);
  p.ll[0] = reinterpret_cast<uint64_t*>(ws + STEP_CONTROL_BYTES + (size_t)2 * p.grid * 8);
  p.ll[1] = p.ll[0] + p.ll_words;
  p.ll[2] = p.ll[1] + p.ll_words;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.grid);
  cfg.blockDim = dim3(kT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, nf4_decode_step_kernel, p);
}

int read_step_error(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_step_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_step_error, &zero, sizeof(int));
  }
  return v;
}

}  // namespace nf4b
