// NF4 GEMM for prefill and batched decode (more than 8 activation rows) on
// the sm_100a tensor cores: tcgen05.mma with TMEM accumulators.
//
// The reference has no large-row kernel: it slices a prompt into 32-row
// launches of the same mma.sync kernel (app/engine/nf4gemv.py:460-478), and
// bitsandbytes itself dequantises the whole weight into a dense GEMM
// (app/engine/nf4gemv.py:10-13). Here one CTA computes a 128-weight-row x BT
// activation-row tile of Y^T (weights on the MMA's M side, activations on its
// N side, so each dequantised weight tile feeds BT rows at once):
//
//   warp 0     TMA producer: X tile [BT x 64] bf16 (128-byte swizzle) and the
//              packed weight tile [128 x 32 B] per 64-wide k block, into a
//              ring_stages<BT>()-deep ring, completion via mbarrier transaction
//              counts; the first ring's weight tiles are requested before the
//              dependency wait (weights are not the previous launch's output).
//   warps 1-2  warp 1 allocates TMEM; one thread of each (of warp 1 only for
//              128- and 256-row tiles) issues 4 x tcgen05.mma (M=128, N=BT, K=16) per
//              k block of its share, into its own fp32 accumulator (BT
//              columns), committing each stage back to the producer and the
//              whole tile to the epilogue.
//   warps 3-18 four groups of four warps, k blocks round-robin over the
//              groups, dequantise: lane l of warp w owns weight row
//              32 (w % 4) + l of the tile; it forms the
//              block's scale (plain fp32, or code2[a8] * absmax2 + offset as two
//              rounded fp32 ops) and writes bf16(NF4[q] * scale) - bit-exact to
//              bitsandbytes' dequantisation - into its row's lane of the A ring
//              in tensor memory (tcgen05.st), which the MMA reads as its A
//              operand: the weights never pass through shared memory, whose
//              bandwidth the X tiles' copies and the MMA's B reads already
//              use (the dequantised tiles never do). After the last k block
//              the same warps read the accumulator back (tcgen05.ld, 32 lanes
//              x 32 columns at a time), round to bf16, apply the epilogue and
//              store Y, through the then idle X ring for split-K and 64-row
//              tiles.
//
// Every mbarrier wait is bounded: a wait that outlives g_gemm_wait_ns (2 s) sets the
// library's device error word and a CTA-wide abort flag, after which every
// role leaves its loop; the producer waits (bounded) for the copies it issued
// and the MMA thread for its last commit, then TMEM is released and the kernel
// returns.

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.cuh"
#include "tmap.cuh"

namespace nf4b {

__device__ int g_device_error = 0;
// Every wait's limit (2 s), and the test hook's switch: when set, the producer
// leaves block 0's activation tile unrequested, so the barrier that copy would
// complete never does and the waits on it run out (set_gemm_debug).
__device__ unsigned long long g_gemm_wait_ns = 2000000000ull;
__device__ int g_gemm_skip_x0 = 0;

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
// DQ groups of four dequantisation/epilogue warps (group g serves k blocks
// g, g + DQ, ...) follow the control warps. Per 64-block each dequantisation thread builds its row's scaled table and
// runs ~170 byte-permute instructions (~1000 cycles per group and block); four
// groups measured faster than two or three, and five or six (more threads,
// fewer registers each) slower again.
// Warps 0-2 are the producer and the MMA issuers; the dequantisation warps
// follow.
constexpr int kControlWarps = 3;
template <int DQ>
constexpr int gemm_threads() { return 32 * kControlWarps + 128 * DQ; }
// MMA issuing threads: each thread's issue loop (barrier wait, fence, four
// MMAs, commit: ~630 cycles per k block, whatever the tile's width) is the
// kernel's serial path for 64-row tiles (batched decode), so those use two,
// in different warps, taking alternate k blocks into two accumulators that
// the epilogue adds (even blocks' sum + odd blocks' sum). Wider tiles keep one:
// with weights streamed cold from HBM a second issuer on 128-row tiles measured
// 3.5% slower at M = 256 (nothing gained with warm weights), and 256-row tiles
// have no tensor memory for a second accumulator.
template <int BT>
__host__ __device__ constexpr int mma_issuers() { return BT <= 64 ? 2 : 1; }
constexpr int kDequantGroups = 4;
// Ring depth: 4 stages (8 for the 64-row tiles, which fit twice as many in
// the same shared memory; deeper rings measured no faster). The depth must be
// a multiple of DQ: group g then meets every phase of its stages in order
// (block j's previous use of stage j % STAGES, block j - STAGES, was the
// group's own), so a parity wait can never be satisfied by the phase two
// rounds back - with more groups than stages it could, and a group would
// read a stale tile.
template <int BT>
__host__ __device__ constexpr int ring_stages() { return BT >= 128 ? 4 : 8; }
// Tensor memory per CTA: the fp32 accumulators (one per MMA issuer, BT
// columns each), then the A ring -
// the dequantised weight tiles, 128 lanes (weight rows) x 32 columns (64 bf16
// or fp16 codes, two per column) per stage, which the MMA reads straight from
// tensor memory, so A never passes through shared memory. Allocated as the
// next power of two.
template <int BT>
__host__ __device__ constexpr uint32_t tmem_cols() {
  return (mma_issuers<BT>() * BT + ring_stages<BT>() * 32) <= 256 ? 256u : 512u;
}
static_assert(2 * 128 + 4 * 32 <= 512 && 2 * 64 + 8 * 32 <= 512 && 256 + 4 * 32 <= 512,
              "accumulators and A ring exceed tensor memory");
static_assert(ring_stages<256>() % kDequantGroups == 0 && ring_stages<128>() % kDequantGroups == 0 &&
                  ring_stages<64>() % kDequantGroups == 0,
              "ring depth must be a multiple of the dequantisation groups");
// A waiting thread asks to be suspended for up to this long per try (it wakes
// when the phase completes): spinning waiters would take issue slots from the
// dequantisation warps (measured 3-4% on the S2-Pro layer at 256-4096 rows).
constexpr uint32_t kSuspendNs = 1000;

template <int BT>
struct __align__(1024) TileSmem {
  static constexpr int STAGES = ring_stages<BT>();
  uint8_t x[STAGES][BT * 128];
  uint8_t w[STAGES][BM * 32];
  float code2[256];
  unsigned long long w_full[STAGES];  // packed weight tile landed (dequantisers wait)
  unsigned long long x_full[STAGES];  // activation tile landed (one dequantisation warp waits)
  unsigned long long a_full[STAGES];  // A stage written and X seen landed (MMA issuer waits)
  unsigned long long mma_done[STAGES];
  unsigned long long accum_full;
  uint32_t tmem_base;
  int abort_flag;
  int last;  // split-K: this CTA finishes its tile
};

// The epilogue stages the fp32 tile [BT][BM] in the X ring.
static_assert(ring_stages<64>() * 64 * 128 >= 64 * BM * 4 && ring_stages<128>() * 128 * 128 >= 128 * BM * 4 &&
                  ring_stages<256>() * 256 * 128 >= 256 * BM * 4,
              "the X ring cannot hold the output tile");
// Each ring (plus 1 KB of alignment slack) fits the 227 KB of shared memory a CTA may use.
static_assert(sizeof(TileSmem<64>) + 1024 <= 232448, "64-row ring too deep");
static_assert(sizeof(TileSmem<128>) + 1024 <= 232448, "128-row ring too deep");
static_assert(sizeof(TileSmem<256>) + 1024 <= 232448, "256-row ring too deep");

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

// Bounded wait on an mbarrier phase. Returns false if the CTA is aborting.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  unsigned long long start = 0;
  for (uint32_t i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity), "n"(kSuspendNs)
        : "memory");
    if (done) return true;
    if ((i & 255u) == 0u) {
      if (*abort_flag) return false;
      const unsigned long long now = globaltimer();
      if (i == 0) {
        start = now;
      } else if (now - start > g_gemm_wait_ns) {
        *abort_flag = 1;
        atomicOr(&g_device_error, 1);
        return false;
      }
    }
  }
}

// Bounded wait for a phase that must complete whether or not the CTA is
// aborting (copies and MMAs already issued): the CTA may not release its
// shared memory or TMEM while they are in flight.
__device__ __forceinline__ void mbar_drain(uint32_t bar, uint32_t parity) {
  unsigned long long start = 0;
  for (uint32_t i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return;
    if ((i & 255u) == 0u) {
      const unsigned long long now = globaltimer();
      if (i == 0) {
        start = now;
      } else if (now - start > g_gemm_wait_ns) {
        atomicOr(&g_device_error, 1);
        return;
      }
    }
  }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// 32 consecutive fp32 columns of this warp's tensor-memory lane quarter.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// The tile's accumulated sums for 32 activation rows (columns c0..c0+31) of
// this warp's 32 weight rows: the first accumulator, plus the second one's
// (at column offset `second`) when two issuers wrote it.
template <int NI>
__device__ __forceinline__ void acc_columns(uint32_t taddr, uint32_t second, bool use_second, float (&a)[32]) {
  uint32_t v[32];
  tmem_ld32(taddr, v);
#pragma unroll
  for (int i = 0; i < 32; ++i) a[i] = __uint_as_float(v[i]);
  if (NI == 2 && use_second) {
    tmem_ld32(taddr + second, v);
#pragma unroll
    for (int i = 0; i < 32; ++i) a[i] = __fadd_rn(a[i], __uint_as_float(v[i]));
  }
}

// K-major, 128-byte-swizzled operand: rows of 128 B, 8-row atoms of 1024 B.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  uint64_t d = (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;             // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
  return d;
}

// kind::f16 instruction descriptor: A and B both bf16 (format 1) or both
// fp16 (format 0), fp32 accumulator.
template <int BT, bool kF16 = false>
__host__ __device__ constexpr uint32_t instr_desc() {
  return (1u << 4)                      // D: fp32
         | ((kF16 ? 0u : 1u) << 7)      // A: bf16 / fp16
         | ((kF16 ? 0u : 1u) << 10)     // B: bf16 / fp16
         | ((uint32_t)(BT >> 3) << 17)  // N
         | ((uint32_t)(BM >> 4) << 24); // M
}

template <int BT, int DQ, bool kSplit, bool kF16 = false>
__global__ void __launch_bounds__(gemm_threads<DQ>(), 1)
    nf4_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_x,
                       const __grid_constant__ CUtensorMap tmap_w, const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  constexpr int STAGES = ring_stages<BT>();
  TileSmem<BT>& sm = *reinterpret_cast<TileSmem<BT>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * BM;
  const int tok0 = blockIdx.y * BT;
  const int KB = p.K / BK;
  // split-K: this CTA's k blocks [kb_lo, kb_lo + nkb)
  const int S = kSplit ? (int)gridDim.z : 1, z = kSplit ? (int)blockIdx.z : 0;
  const int kb_lo = kSplit ? (int)((long long)KB * z / S) : 0;
  const int nkb = kSplit ? (int)((long long)KB * (z + 1) / S) - kb_lo : KB;
  volatile int* abort_flag = &sm.abort_flag;

  if (tid == 0) {
    sm.abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&sm.w_full[s]), 1);
      mbar_init(smem_u32(&sm.x_full[s]), 1);
      mbar_init(smem_u32(&sm.a_full[s]), 4);
      mbar_init(smem_u32(&sm.mma_done[s]), 1);
    }
    mbar_init(smem_u32(&sm.accum_full), mma_issuers<BT>());
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&sm.tmem_base)),
                 "r"(tmem_cols<BT>())
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = sm.tmem_base;
  // The next launch may be scheduled now: its CTAs take the SMs this grid
  // leaves idle (a partial wave; they cannot share an SM with this kernel's
  // CTAs) and run their prologue - weight copies and their dequantisation for
  // a GEMM - before their own dependency wait, which waits for this grid to
  // complete (measured 1-3% on the S2-Pro layer from M = 32 to 1024).
  pdl_launch_dependents();

  // Only X, Y, the epilogue operand and the split-K scratch belong to the
  // stream's previous work: the producer requests the first weight tiles
  // before its dependency wait, and the dequantisation warps wait only
  // before their epilogue.
  if (warp == 0) {
    if (lane == 0) {
      int issued_w = 0, issued = 0;
      auto load_w = [&](int i) {
        const uint32_t wbar = smem_u32(&sm.w_full[i % STAGES]);
        mbar_expect_tx(wbar, BM * 32);
        tma_load_2d(smem_u32(sm.w[i % STAGES]), &tmap_w, (kb_lo + i) * (BK / 2), n0, wbar);
        issued_w = i + 1;
      };
      for (int i = 0; i < nkb && i < STAGES; ++i) load_w(i);
      pdl_wait();
      const bool skip_x0 = g_gemm_skip_x0 != 0;  // test hook only
      for (int i = 0; i < nkb; ++i) {
        const int s = i % STAGES;
        if (i >= STAGES) {
          if (!mbar_wait(smem_u32(&sm.mma_done[s]), ((i / STAGES) - 1) & 1, abort_flag)) break;
          // the small weight tile first, on its own barrier, so that its
          // dequantisation starts before the activation tile has landed
          load_w(i);
        }
        if (!(skip_x0 && i == 0)) {
          const uint32_t xbar = smem_u32(&sm.x_full[s]);
          mbar_expect_tx(xbar, BT * 128);
          tma_load_2d(smem_u32(sm.x[s]), &tmap_x, (kb_lo + i) * BK, tok0, xbar);
        }
        issued = i + 1;
      }
      // every copy issued has landed before the CTA can exit (immediate on the
      // normal path: the consumers have waited for them all)
      for (int i = issued_w > STAGES ? issued_w - STAGES : 0; i < issued_w; ++i)
        mbar_drain(smem_u32(&sm.w_full[i % STAGES]), (i / STAGES) & 1);
      for (int i = issued > STAGES ? issued - STAGES : 0; i < issued; ++i)
        mbar_drain(smem_u32(&sm.x_full[i % STAGES]), (i / STAGES) & 1);
    }
  } else if (warp < kControlWarps) {
    constexpr int NI = mma_issuers<BT>();
    const int j = warp - 1;  // issuer j takes k blocks j, j + NI, ... into accumulator j
    if (lane == 0 && j < NI) {
      constexpr uint32_t idesc = instr_desc<BT, kF16>();
      // This thread's loop is the kernel's serial path (every barrier wait,
      // MMA issue and commit here costs tens to ~150 cycles even when its
      // operands are long ready), so it waits on ONE barrier per k block:
      // a_full completes when the block's group has written the A stage and
      // one of its warps has seen the X tile land.
      const uint32_t d_tmem = tmem + (uint32_t)(j * BT);
      for (int i = j; i < nkb; i += NI) {
        const int s = i % STAGES;
        if (!mbar_wait(smem_u32(&sm.a_full[s]), (i / STAGES) & 1, abort_flag)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        // A: 128 lanes x 8 columns (16 codes) of the stage in tensor memory per
        // MMA; B: the X stage, 32 bytes further per 16-wide k step (+2 in the
        // descriptor's 16-byte address field, which cannot carry: shared
        // addresses are below 2^18)
        const uint32_t a_tmem = tmem + (uint32_t)(NI * BT) + (uint32_t)s * 32u;
        const uint64_t bd = smem_desc(smem_u32(sm.x[s]));
        asm volatile(
            "{\n\t.reg .pred p, q;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "setp.eq.b32 q, %4, %4;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%5], %6, %3, q;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%7], %8, %3, q;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%9], %10, %3, q;\n\t}" ::"r"(d_tmem),
            "r"(a_tmem), "l"(bd), "r"(idesc), "r"((uint32_t)(i - j)), "r"(a_tmem + 8u), "l"(bd + 2), "r"(a_tmem + 16u),
            "l"(bd + 4), "r"(a_tmem + 24u), "l"(bd + 6)
            : "memory");
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::
                         "r"(smem_u32(&sm.mma_done[s]))
                     : "memory");
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::
                       "r"(smem_u32(&sm.accum_full))
                   : "memory");
      // every MMA issued has completed before TMEM is released
      mbar_drain(smem_u32(&sm.accum_full), 0);
    }
  } else {
    // Dequantise: lane l of a warp owns weight row r = 32 (warp % 4) + l of the
    // tile - its tensor-memory lane, the only lane quarter the warp may write.
    const int grp = (warp - kControlWarps) >> 2;
    const int r = (warp & 3) * 32 + lane;
    const int row = n0 + r;
    const bool valid = row < p.N;
    const uint32_t a_lane = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(mma_issuers<BT>() * BT);
    // The block scale's global loads run one of this group's k blocks ahead,
    // so their latency hides under the previous block's dequantisation.
    uint32_t code_next = 0;
    float am_next = 0.f;
    auto fetch_scale = [&](int i) {
      if (valid && i < nkb) {
        const size_t b = ((size_t)row * p.K + (size_t)(kb_lo + i) * BK) >> p.bs_shift;
        if (p.nested) {
          code_next = __ldg(p.a8 + b);
          am_next = __ldg(p.absmax + (b >> p.bs2_shift));
        } else {
          am_next = __ldg(p.absmax + b);
        }
      }
    };
    fetch_scale(grp);
    // code2 (a weight table) into shared memory while the first copies land;
    // the dequantisation threads alone meet at this barrier
    if (p.nested)
      for (int i = tid - 32 * kControlWarps; i < 256; i += DQ * 128) sm.code2[i] = p.code2[i];
    asm volatile("bar.sync 1, %0;" ::"n"(DQ * 128) : "memory");
    // Row r's 32 packed bytes, its two 16-byte halves read in an order that
    // alternates every 4 rows: the warp's 16-byte reads then cover all 8
    // bank groups of each 128 bytes (no 2-way conflict).
    const int hfirst = (r >> 2) & 1;
    for (int i = grp; i < nkb; i += DQ) {
      const int s = i % STAGES;
      const uint32_t code = code_next;
      const float am = am_next;
      fetch_scale(i + DQ);
      const float scale = !valid ? 0.f : p.nested ? nested_scale(sm.code2[code], am, p.offset) : am;
      if (!mbar_wait(smem_u32(&sm.w_full[s]), (i / STAGES) & 1, abort_flag)) break;
      // the stage's previous MMAs completed before this tile's copy was issued:
      // order the tensor-memory store below after that
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint4* wp = reinterpret_cast<const uint4*>(sm.w[s] + r * 32);
      const uint4 ua = wp[hfirst], ub = wp[hfirst ^ 1];
      const uint4 u0 = hfirst ? ub : ua, u1 = hfirst ? ua : ub;
      const uint32_t words[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
      const ScaledLut lut = scaled_lut<kF16>(scale);
      // the row's 64 codes as 32 pairs in k order -> columns 0..31 of its lane
      uint32_t o[32];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t q4[4];
        lut_dequant8(lut, words[c], q4);
#pragma unroll
        for (int e = 0; e < 4; ++e) o[4 * c + e] = q4[e];
      }
      asm volatile(
          "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
          "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
          "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(a_lane + (uint32_t)s * 32u),
          "r"(o[0]), "r"(o[1]), "r"(o[2]), "r"(o[3]), "r"(o[4]), "r"(o[5]), "r"(o[6]), "r"(o[7]), "r"(o[8]),
          "r"(o[9]), "r"(o[10]), "r"(o[11]), "r"(o[12]), "r"(o[13]), "r"(o[14]), "r"(o[15]), "r"(o[16]),
          "r"(o[17]), "r"(o[18]), "r"(o[19]), "r"(o[20]), "r"(o[21]), "r"(o[22]), "r"(o[23]), "r"(o[24]),
          "r"(o[25]), "r"(o[26]), "r"(o[27]), "r"(o[28]), "r"(o[29]), "r"(o[30]), "r"(o[31])
          : "memory");
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      // the group's first warp also sees the block's X tile land, so that
      // a_full alone tells the MMA issuer both operands are ready
      if ((warp & 3) == 0 && !mbar_wait(smem_u32(&sm.x_full[s]), (i / STAGES) & 1, abort_flag)) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&sm.a_full[s]));
    }

    // Epilogue. TMEM lane quarter (warp % 4) holds weight rows 32q..32q+31;
    // each warp reads its column blocks (32 activation rows) with tcgen05.ld.
    // Unsplit 128- and 256-row tiles store Y straight from those registers
    // (a warp's store is 32 consecutive outputs of one activation row). The
    // split-K partial sums and 64-row tiles go through the X ring (free once
    // every MMA has completed) instead: stored transposed as fp32 [BT][BM],
    // read back along n four outputs per thread and written as whole 8-byte
    // (16-byte) runs of each activation row (measured on the S2-Pro
    // projections: 2-14% faster on those launches, 7-11% slower on unsplit
    // 128- and 256-row tiles).
    float* stage = reinterpret_cast<float*>(&sm.x[0][0]);
    pdl_wait();
    constexpr bool kStaged = kSplit || BT == 64;
    if (!kStaged) {
      if (mbar_wait(smem_u32(&sm.accum_full), 0, abort_flag)) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int q = warp & 3;
        const int n = n0 + q * 32 + lane;
        for (int cb = grp; cb < BT / 32; cb += DQ) {
          float a[32];
          acc_columns<mma_issuers<BT>()>(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(cb * 32), (uint32_t)BT,
                                         nkb > 1, a);
          if (n < p.N) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int tok = tok0 + cb * 32 + i;
              if (tok < p.M) {
                const size_t o = (size_t)tok * p.N + n;
                p.y[o] = epilogue<kF16>(a[i], p.epi, p.operand, o);
              }
            }
          }
        }
      }
    } else {
    if (mbar_wait(smem_u32(&sm.accum_full), 0, abort_flag)) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int q = warp & 3;
      for (int cb = grp; cb < BT / 32; cb += DQ) {
        float a[32];
        acc_columns<mma_issuers<BT>()>(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(cb * 32), (uint32_t)BT,
                                       nkb > 1, a);
        float* col = stage + (size_t)(cb * 32) * BM + q * 32 + lane;
#pragma unroll
        for (int i = 0; i < 32; ++i) col[i * BM] = a[i];
      }
    }
    // every dequantisation thread reaches this barrier, aborting or not
    asm volatile("bar.sync 1, %0;" ::"n"(DQ * 128) : "memory");
    if (!*abort_flag) {
      const int t = tid - 32 * kControlWarps;
      const bool vec = (p.N & 3) == 0 && (kSplit || (((uintptr_t)p.y | (uintptr_t)p.operand) & 7) == 0);
      float* part = kSplit ? p.partial + (size_t)z * p.M * p.N : nullptr;
      for (int e = t; e < BT * (BM / 4); e += DQ * 128) {
        const int tok = tok0 + e / (BM / 4), n = n0 + (e % (BM / 4)) * 4;
        if (tok >= p.M || n >= p.N) continue;
        const float4 a = *reinterpret_cast<const float4*>(stage + (size_t)e * 4);
        const size_t o = (size_t)tok * p.N + n;
        if (vec && kSplit) {
          __stcg(reinterpret_cast<float4*>(part + o), a);
        } else if (vec) {
          float opv[4] = {0.f, 0.f, 0.f, 0.f};
          if (p.epi != NF4B_EPI_NONE) {
            const uint2 ov = *reinterpret_cast<const uint2*>(p.operand + o);
            opv[0] = act2f<kF16>((uint16_t)(ov.x & 0xFFFFu));
            opv[1] = act2f<kF16>((uint16_t)(ov.x >> 16));
            opv[2] = act2f<kF16>((uint16_t)(ov.y & 0xFFFFu));
            opv[3] = act2f<kF16>((uint16_t)(ov.y >> 16));
          }
          const uint32_t y0 = epilogue_value<kF16>(a.x, p.epi, opv[0]), y1 = epilogue_value<kF16>(a.y, p.epi, opv[1]);
          const uint32_t y2 = epilogue_value<kF16>(a.z, p.epi, opv[2]), y3 = epilogue_value<kF16>(a.w, p.epi, opv[3]);
          *reinterpret_cast<uint2*>(p.y + o) = make_uint2(y0 | (y1 << 16), y2 | (y3 << 16));
        } else {
          const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            if (n + c >= p.N) break;
            if (kSplit)
              __stcg(part + o + c, av[c]);
            else
              p.y[o + c] = epilogue<kF16>(av[c], p.epi, p.operand, o + c);
          }
        }
      }
    }
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  if (kSplit) __threadfence();  // this thread's partial stores, before the tile's count below
  if (warp < kControlWarps) pdl_wait();  // the split's counters below belong to the previous work as well
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(tmem_cols<BT>())
                 : "memory");
  }
  if (kSplit) {
    // The tile's last CTA to finish sums the S partials in split order
    // (deterministic) and stores Y; the counter is re-zeroed for the next launch.
    int* ctr = p.counters + blockIdx.y * gridDim.x + blockIdx.x;
    if (tid == 0) {
      __threadfence();
      const int old = atomicAdd(ctr, 1);
      sm.last = (old == S - 1);
      if (sm.last) *ctr = 0;
    }
    __syncthreads();
    if (!sm.last || *abort_flag) return;
    __threadfence();
    // The tile's BT x 128 sums, read as float4 runs along n (when n_out % 4 == 0)
    // with every split's loads of a thread's elements issued before the
    // in-order sums: a few L2 round trips for the whole tile.
    const size_t MN = (size_t)p.M * p.N;
    constexpr int T = gemm_threads<DQ>();
    if ((p.N & 3) == 0) {
      constexpr int V = 2;  // float4s per thread per split in flight
      for (int base = tid; base < BT * (BM / 4); base += V * T) {
        float4 acc[V];
        size_t o[V];
        bool live[V];
#pragma unroll
        for (int e = 0; e < V; ++e) {
          const int idx = base + e * T;
          const int tok = tok0 + idx / (BM / 4), n = n0 + (idx % (BM / 4)) * 4;
          live[e] = idx < BT * (BM / 4) && tok < p.M && n < p.N;
          o[e] = live[e] ? (size_t)tok * p.N + n : 0;
          acc[e] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        for (int z0 = 0; z0 < S; z0 += 4) {
          float4 v[4][V];
#pragma unroll
          for (int zz = 0; zz < 4; ++zz)
#pragma unroll
            for (int e = 0; e < V; ++e)
              v[zz][e] = (live[e] && z0 + zz < S)
                             ? __ldcg(reinterpret_cast<const float4*>(p.partial + (z0 + zz) * MN + o[e]))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int zz = 0; zz < 4; ++zz)
            if (z0 + zz < S)
#pragma unroll
              for (int e = 0; e < V; ++e) {
                acc[e].x += v[zz][e].x;
                acc[e].y += v[zz][e].y;
                acc[e].z += v[zz][e].z;
                acc[e].w += v[zz][e].w;
              }
        }
#pragma unroll
        for (int e = 0; e < V; ++e)
          if (live[e]) {
            const float a[4] = {acc[e].x, acc[e].y, acc[e].z, acc[e].w};
#pragma unroll
            for (int c = 0; c < 4; ++c) p.y[o[e] + c] = epilogue<kF16>(a[c], p.epi, p.operand, o[e] + c);
          }
      }
      return;
    }
    // four elements per thread in flight, each with all its splits' loads issued
    // before the in-order sum
    for (int base = tid; base < BT * BM; base += 4 * T) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      size_t o[4];
      bool live[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int idx = base + e * T;
        const int tok = tok0 + idx / BM, n = n0 + idx % BM;
        live[e] = idx < BT * BM && tok < p.M && n < p.N;
        o[e] = live[e] ? (size_t)tok * p.N + n : 0;
      }
      for (int z0 = 0; z0 < S; z0 += 4) {
        float v[4][4];
#pragma unroll
        for (int zz = 0; zz < 4; ++zz)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            v[zz][e] = (live[e] && z0 + zz < S) ? __ldcg(p.partial + (z0 + zz) * MN + o[e]) : 0.f;
#pragma unroll
        for (int zz = 0; zz < 4; ++zz)
          if (z0 + zz < S)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[e] += v[zz][e];
      }
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (live[e]) p.y[o[e]] = epilogue<kF16>(acc[e], p.epi, p.operand, o[e]);
    }
  }
}

template <int BT, bool kSplit, bool kF16 = false>
cudaError_t launch_bt(const GemmParams& p, cudaStream_t stream) {
  CUtensorMap mx, mw;
  if (!make_map_2d(&mx, kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, p.x, (uint64_t)p.K, (uint64_t)p.M,
                   (uint64_t)p.K * 2, BK, BT, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if (!make_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.packed, (uint64_t)p.K / 2, (uint64_t)p.N,
                   (uint64_t)p.K / 2, BK / 2, BM, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  const size_t smem = sizeof(TileSmem<BT>) + 1024;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(nf4_gemm_tc_kernel<BT, kDequantGroups, kSplit, kF16>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.N + BM - 1) / BM, (p.M + BT - 1) / BT, kSplit ? p.splits : 1);
  cfg.blockDim = dim3(gemm_threads<kDequantGroups>());
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, nf4_gemm_tc_kernel<BT, kDequantGroups, kSplit, kF16>, mx, mw, p);
}

}  // namespace


// Tile rows (BT) and k splits of a GEMM, from a cost model fitted to a sweep of
// the S2-Pro projections (6144x2560, 2560x4096, 9728x2560, 2560x9728) at 32..4096
// rows over BT in {64, 128, 256} and 1..8 splits: a CTA costs ~10 k-block
// times of fixed work (pipeline fill, epilogue) plus its k blocks (relative
// cost 0.8, 1, 1 per k block for 64-, 128-, 256-row tiles: the MMA issue loop
// and the dequantisation, not the tile's MMA width, set a k block's time);
// CTAs beyond one per SM run in further rounds; each split adds its partial
// sums' write and reduction (1.5, 3, 15 k-block times). On that sweep its pick
// is the fastest measured (bt, splits) or within 7% of it for every shape and
// row count (e.g. 2560x9728: 6 splits of 64-row tiles at M = 32-64, 3 splits
// of 128-row tiles at M = 256, unsplit 256-row tiles from M = 1024; the
// 9728-row gate and up projections unsplit, one CTA per tile).
struct GemmShape {
  int bt, splits;
};

static GemmShape gemm_choose(int N, int M, int K, int sms) {
  const long long tn = (N + BM - 1) / BM;
  const int KB = K / BK;
  const int bts[3] = {64, 128, 256};
  const double cost_kb[3] = {0.8, 1.0, 1.0}, cost_split[3] = {1.5, 3.0, 15.0};
  const int splits[6] = {1, 2, 3, 4, 6, 8};
  GemmShape best = {64, 1};
  double best_t = 1e30;
  for (int bi = 0; bi < 3; ++bi) {
    const int bt = bts[bi];
    if (bt > 64 && M <= bt / 2) continue;  // a tile at most half full
    const long long tiles = tn * ((M + bt - 1) / bt);
    for (int si = 0; si < 6; ++si) {
      const int sp = splits[si];
      if (sp > 1 && (KB / sp < 4 || tiles * (long long)sizeof(int) > (long long)GEMM_COUNTER_BYTES)) continue;
      const long long ctas = tiles * sp;
      const long long rounds = (ctas + sms - 1) / sms;
      const double t = (double)rounds * ((double)((KB + sp - 1) / sp) * cost_kb[bi] + 10.0) +
                       (sp > 1 ? sp * cost_split[bi] : 0.0);
      if (t < best_t - 1e-9) {
        best_t = t;
        best = {bt, sp};
      }
    }
  }
  return best;
}

int gemm_bt(int N, int M, int K, int sms) { return gemm_choose(N, M, K, sms).bt; }

int gemm_splits(int N, int M, int K, int sms) { return gemm_choose(N, M, K, sms).splits; }

size_t gemm_workspace_bytes(int N, int M, int K, int sms) {
  const int s = gemm_splits(N, M, K, sms);
  return s > 1 ? GEMM_COUNTER_BYTES + (size_t)s * M * N * sizeof(float) : 0;
}

template <bool kF16>
static cudaError_t launch_gemm_act(const GemmParams& p, cudaStream_t stream) {
  const int bt = p.bt;
  if (bt == 64)
    return p.splits > 1 ? launch_bt<64, true, kF16>(p, stream) : launch_bt<64, false, kF16>(p, stream);
  if (bt == 128)
    return p.splits > 1 ? launch_bt<128, true, kF16>(p, stream) : launch_bt<128, false, kF16>(p, stream);
  return p.splits > 1 ? launch_bt<256, true, kF16>(p, stream) : launch_bt<256, false, kF16>(p, stream);
}

cudaError_t launch_gemm_tc(const GemmParams& p, cudaStream_t stream) {
  return p.f16 ? launch_gemm_act<true>(p, stream) : launch_gemm_act<false>(p, stream);
}

int set_gemm_debug(int skip_x0, unsigned long long wait_ns) {
  if (cudaMemcpyToSymbol(g_gemm_skip_x0, &skip_x0, sizeof(int)) != cudaSuccess) return -1;
  if (cudaMemcpyToSymbol(g_gemm_wait_ns, &wait_ns, sizeof(wait_ns)) != cudaSuccess) return -1;
  return 0;
}

int read_device_error(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
  }
  return v;
}

}  // namespace nf4b
