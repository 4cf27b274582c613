// The C ABI of libnf4b200.so (declared in include/nf4b200.h).
//
// Every entry point validates its arguments on the host and returns a status
// instead of throwing: shape, alignment and dtype problems are reported before
// anything is launched, so a caller can decline and fall back exactly where the
// reference returns None (app/engine/nf4gemv.py:315-376, :436-455). A launch
// failure returns NF4B_ERR_LAUNCH, the analogue of the reference's RuntimeError
// on a non-zero cuLaunchKernel status (app/engine/nf4gemv.py:476-477).

#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"
#include "kernels.cuh"
#include "tmap.cuh"

namespace nf4b {
int read_device_error(int clear);
int set_gemm_debug(int skip_x0, unsigned long long wait_ns);
int read_gemv_error(int clear);
int read_attn_error(int clear);
}

using namespace nf4b;

namespace {
int fail(int code, const char* fmt, ...);
}

namespace nf4b {
// Record `msg` as this thread's last error and return `code` (for entry points
// defined in other files).
int report_error(int code, const char* msg) { return fail(code, "%s", msg); }
}  // namespace nf4b

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int ok() {
  g_err[0] = '\0';
  return NF4B_OK;
}

bool is_pow2(int v) { return v > 0 && (v & (v - 1)) == 0; }
int log2i(int v) {
  int s = 0;
  while ((1 << s) < v) ++s;
  return s;
}
bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
// Rotary tables are read one element at a time: 4-byte fp32 or 2-byte fp16/bf16.
bool freqs_aligned(const void* f, int freqs_dtype) { return aligned(f, freqs_dtype == NF4B_F32 ? 4 : 2); }
// Device int64 scalars and vectors (positions, step counters, token ids); null passes.
bool i64_aligned(const int64_t* p) { return aligned(p, 8); }

int check_device() {
  static int checked[64] = {};  // 0 unknown, 1 ok, -1 bad
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(NF4B_ERR_DEVICE, "no current CUDA device");
  if (checked[dev] == 0) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    checked[dev] = (major == 10 && minor == 0) ? 1 : -1;
  }
  if (checked[dev] < 0)
    return fail(NF4B_ERR_DEVICE, "device %d is not sm_100 (this library is built for sm_100a)", dev);
  return NF4B_OK;
}

int check_weight(const nf4b_weight* w) {
  if (w == nullptr || w->packed == nullptr || w->absmax == nullptr)
    return fail(NF4B_ERR_ARG, "weight descriptor or its packed/absmax pointer is null");
  if (w->n_out <= 0 || w->k_in <= 0) return fail(NF4B_ERR_SHAPE, "empty weight %dx%d", w->n_out, w->k_in);
  if (!is_pow2(w->blocksize) || w->blocksize < 64)
    return fail(NF4B_ERR_SHAPE, "blocksize %d is not a power of two >= 64", w->blocksize);
  if (w->k_in % w->blocksize || w->k_in % 64)
    return fail(NF4B_ERR_SHAPE, "in_features %d is not a multiple of 64 and of the blocksize %d",
                w->k_in, w->blocksize);
  if (!aligned(w->packed, 16)) return fail(NF4B_ERR_ALIGN, "packed weight is not 16-byte aligned");
  if (w->nested) {
    if (w->absmax_code == nullptr || w->code2 == nullptr)
      return fail(NF4B_ERR_ARG, "nested weight without absmax codes or code2 table");
    if (!is_pow2(w->blocksize2))
      return fail(NF4B_ERR_SHAPE, "second-level blocksize %d is not a power of two", w->blocksize2);
  }
  return NF4B_OK;
}

int launch_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return fail(NF4B_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  return ok();
}

// The pair GEMV reads two adjacent 64-block scales at once (a 2-byte code pair
// or an 8-byte fp32 pair) and assumes an even block and its successor share a
// second-level block.
// The byte ranges of an L2 prefetch hint: the packed codes and the first-level
// scales of each named weight (16-byte aligned, whole 16-byte chunks).
void prefetch_ranges(const nf4b_gemm_opts* opts, PrefetchHint* h) {
  for (int i = 0; i < 4; ++i) {
    h->ptr[i] = nullptr;
    h->bytes[i] = 0;
  }
  if (opts == nullptr) return;
  const nf4b_weight* ws[2] = {opts->prefetch_next, opts->prefetch_next2};
  for (int i = 0; i < 2; ++i) {
    const nf4b_weight* nx = ws[i];
    if (nx == nullptr || nx->packed == nullptr || !aligned(nx->packed, 16) || nx->n_out <= 0 ||
        nx->k_in <= 0 || nx->blocksize <= 0)
      continue;
    h->ptr[2 * i] = nx->packed;
    h->bytes[2 * i] = ((long long)nx->n_out * nx->k_in / 2) & ~15LL;
    const long long nb = (long long)nx->n_out * nx->k_in / nx->blocksize;
    const void* sc = nx->nested ? (const void*)nx->absmax_code : (const void*)nx->absmax;
    if (sc != nullptr && aligned(sc, 16)) {
      h->ptr[2 * i + 1] = static_cast<const uint8_t*>(sc);
      h->bytes[2 * i + 1] = (nb * (nx->nested ? 1 : 4)) & ~15LL;
    }
  }
}

// 128-code sub-units per pair-kernel unit: 2 when a unit's four 64-blocks
// start at a multiple of 4 (k_in % 256 == 0) so their scale data is one
// aligned copy - nested with second-level blocks of >= 4 (one shared
// second-level scale), or fp32 scales 16-byte aligned - and x can be staged.
int pair_su(const nf4b_weight* w, int rows) {
  if (w->blocksize != 64 || w->k_in % 256 || (long long)rows * w->k_in * 2 > GEMV_PAIR_X_MAX) return 1;
  if (w->nested) return w->blocksize2 >= 4 ? 2 : 1;
  return aligned(w->absmax, 16) ? 2 : 1;
}

bool use_pairs(const nf4b_weight* w, int rows) {
  if (rows > 4 || w->k_in % 128) return false;
  // The pair kernel copies scales with 4- and 8-byte cp.async: the 8-bit codes
  // as 4-byte aligned windows, fp32 scales at their natural alignment (paired
  // when blocks are 64 codes), and the 1 KB code2 table in 16-byte pieces.
  if (w->nested)
    return aligned(w->absmax_code, 4) && aligned(w->absmax, 4) && aligned(w->code2, 16) &&
           w->blocksize2 >= (w->blocksize == 64 ? 2 : 1);
  return aligned(w->absmax, w->blocksize == 64 ? 8 : 4);
}

bool reg_eligible(const nf4b_weight* w, const nf4b_weight* w3, int rows);

size_t gemv_workspace_bytes(const nf4b_weight* w, int rows, int sms) {
  GemvPlan a;
  gemv_plan(w->n_out, w->k_in, rows, sms, false, &a);
  size_t bytes = a.partial_bytes;
  // the pair or register-fed kernel may serve this call, plain or gated
  const int su_max = reg_eligible(w, nullptr, rows) ? 2 : (rows <= 4 && w->k_in % 128 == 0) ? pair_su(w, rows) : 0;
  for (int gated = 0; gated < 2; ++gated)
    for (int su = 1; su <= su_max; ++su) {
      GemvPlan b;
      gemv_plan(w->n_out, w->k_in, rows, sms, true, &b, gated != 0, su);
      if (b.partial_bytes > bytes) bytes = b.partial_bytes;
    }
  return GEMV_COUNTER_BYTES + bytes;
}

int current_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  return gemv_sm_count(dev);
}

// The activation type named by the options: 0 / NF4B_BF16 = bf16 (the
// default of zeroed options), NF4B_F16 = fp16. Returns the status.
int act_type(const nf4b_gemm_opts* opts, bool* f16) {
  *f16 = false;
  if (opts == nullptr || opts->dtype == 0 || opts->dtype == NF4B_BF16) return NF4B_OK;
  if (opts->dtype != NF4B_F16) return fail(NF4B_ERR_DTYPE, "unknown activation dtype %d", opts->dtype);
  *f16 = true;
  return NF4B_OK;
}

// Whether the register-fed pair GEMV serves this weight (pair) at `rows`:
// 1..GEMV_REG_MAX_ROWS rows whose x fits its shared-memory staging,
// blocksize-64 units of 256 codes with their scale data in one aligned copy
// (nested: the pair kernel's alignment, second-level blocks of >= 4; plain:
// 16-byte aligned fp32 scales), 32-byte aligned packed codes.
bool reg_eligible(const nf4b_weight* w, const nf4b_weight* w3, int rows) {
  auto one = [&](const nf4b_weight* v) {
    if (v->blocksize != 64 || v->k_in % 256 || !aligned(v->packed, 32) ||
        (long long)v->n_out * (v->k_in / 64) >= (1LL << 31))
      return false;
    if (v->nested)
      return aligned(v->absmax_code, 4) && aligned(v->absmax, 4) && aligned(v->code2, 16) && v->blocksize2 >= 4;
    return aligned(v->absmax, 16);
  };
  return rows >= 1 && rows <= GEMV_REG_MAX_ROWS && (long long)rows * w->k_in * 2 <= GEMV_REG_X_MAX && one(w) &&
         (w3 == nullptr || one(w3));
}

// One GEMV launch (rows <= GEMV_MAX_ROWS): plain, or the gated pair (w, w3)
// of the pair kernel. Arguments already checked by the caller except the
// workspace and the GEMV-specific limits.
int gemv_call(const nf4b_weight* w, const nf4b_weight* w3, const void* x, void* y, int rows, int epi,
              const void* operand, void* workspace, size_t workspace_bytes, const nf4b_gemm_opts* opts,
              cudaStream_t s, const nf4b_rope_kv* rk = nullptr) {
  if ((long long)(w->n_out + 15) / 16 > GEMV_MAX_TILES)
    return fail(NF4B_ERR_SHAPE, "n_out %d exceeds the GEMV's %lld-row limit", w->n_out, GEMV_MAX_TILES * 16);
  const bool gated = w3 != nullptr;
  // the register-fed kernel (1..8 rows) where it applies, else the TMA-ring
  // pair kernel (1..4 rows), else the block kernel
  const bool reg = reg_eligible(w, w3, rows);
  const bool pairs = reg || use_pairs(w, rows);
  if (gated && !(reg || (pairs && use_pairs(w3, rows))))
    return fail(NF4B_ERR_SHAPE,
                "the gated GEMV serves 1..8 rows on the register-fed kernel (blocksize 64, k_in %% 256 == 0) or 1..4 "
                "rows with k_in %% 128 == 0 (got %d rows, k_in %d)",
                rows, w->k_in);
  const int sms = current_sm_count();
  const int su = reg ? 2
                     : pairs ? (gated ? (pair_su(w, rows) == 2 && pair_su(w3, rows) == 2 ? 2 : 1) : pair_su(w, rows))
                             : 1;
  GemvPlan plan;
  gemv_plan(w->n_out, w->k_in, rows, sms, pairs, &plan, gated, su);
  const size_t need = gemv_workspace_bytes(w, rows, sms);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(NF4B_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need,
                workspace ? workspace_bytes : (size_t)0);
  if (!aligned(workspace, 256)) return fail(NF4B_ERR_ALIGN, "workspace is not 256-byte aligned");
  GemvParams p = {};
  p.packed = w->packed;
  p.a8 = w->absmax_code;
  p.absmax = w->absmax;
  p.code2 = w->code2;
  p.offset = w->offset;
  p.packed3 = gated ? w3->packed : nullptr;
  p.a8_3 = gated ? w3->absmax_code : nullptr;
  p.absmax3 = gated ? w3->absmax : nullptr;
  p.code2_3 = gated && w3->nested ? w3->code2 : nullptr;
  p.offset3 = gated ? w3->offset : 0.f;
  p.gated = gated ? 1 : 0;
  p.su = su;
  // The register-fed pair kernel reads 32-byte pieces of the packed weights.
  p.reg = reg ? 1 : 0;
  bool f16 = false;
  int st = act_type(opts, &f16);
  if (st) return st;
  if (f16 && (!p.reg || rk != nullptr))
    return fail(NF4B_ERR_SHAPE, "fp16 is served here on the register-fed decode GEMV only (1..8 rows, blocksize 64, "
                                "k_in %% 256 == 0, 32-byte aligned packed codes)");
  p.f16 = f16 ? 1 : 0;
  if (rk != nullptr) {
    if (!p.reg || gated || rows != 1 || epi != NF4B_EPI_NONE)
      return fail(NF4B_ERR_SHAPE, "the fused rotary store serves one row on the register-fed decode GEMV");
    p.rk_freqs = rk->freqs;
    p.rk_ftype = rk->freqs_dtype;
    p.rk_pos = rk->pos;
    p.rk_q = static_cast<uint16_t*>(rk->q_out);
    p.rk_k = static_cast<uint16_t*>(rk->k_cache);
    p.rk_v = static_cast<uint16_t*>(rk->v_cache);
    p.rk_nh = rk->n_head;
    p.rk_nkv = rk->n_kv;
    p.rk_max_len = rk->max_len;
  }
  p.x_staged = (reg || (pairs && (long long)rows * w->k_in * 2 <= GEMV_PAIR_X_MAX)) ? 1 : 0;
  p.norm_w = opts ? static_cast<const uint16_t*>(opts->norm_weight) : nullptr;
  p.norm_eps = opts ? opts->norm_eps : 0.f;
  if (p.norm_w != nullptr && !p.x_staged)
    return fail(NF4B_ERR_SHAPE, "a fused RMSNorm needs x staged (1..4 rows, k_in %% 128 == 0, rows * k_in * 2 <= %d)",
                GEMV_PAIR_X_MAX);
  if (p.norm_w != nullptr && !aligned(p.norm_w, 2)) return fail(NF4B_ERR_ALIGN, "norm weight not 2-byte aligned");
  p.N = w->n_out;
  p.K = w->k_in;
  p.nested = w->nested ? 1 : 0;
  p.bs_shift = log2i(w->blocksize);
  p.bs2_shift = w->nested ? log2i(w->blocksize2) : 0;
  p.x = static_cast<const uint16_t*>(x);
  p.y = static_cast<uint16_t*>(y);
  p.operand = static_cast<const uint16_t*>(operand);
  p.M = rows;
  p.epi = gated ? NF4B_EPI_NONE : epi;
  p.counters = static_cast<int*>(workspace);
  p.partial = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + plan.counter_bytes);
  p.units = plan.units;
  p.warps_total = plan.warps_total;
  p.uq = (int)(plan.units / plan.warps_total);
  p.ur = (int)(plan.units % plan.warps_total);
  p.blocks_per_tile = plan.blocks_per_tile;
  prefetch_ranges(opts, &p.pf);
  return launch_status(launch_gemv(p, plan.grid, pairs, s), "nf4 gemv launch");
}

}  // namespace

extern "C" {

int nf4b_version(void) { return 200; }

const char* nf4b_last_error(void) { return g_err; }

int nf4b_device_error(int clear) {
  const int gemm = read_device_error(clear), gemv = read_gemv_error(clear), attn = read_attn_error(clear);
  const int step = read_step_error(clear);
  if (gemm < 0 || gemv < 0 || attn < 0 || step < 0) return -1;
  return (gemm ? 1 : 0) | (gemv ? 2 : 0) | (attn ? 4 : 0) | (step ? 8 : 0);
}

size_t nf4b_gemm_workspace_size(const nf4b_weight* w, int rows) {
  if (w == nullptr || rows <= 0 || w->n_out <= 0 || w->k_in <= 0) return 0;
  const int sms = current_sm_count();
  if (rows > GEMV_MAX_ROWS) return gemm_workspace_bytes(w->n_out, rows, w->k_in, sms);
  // 1..32 rows: the GEMV's, or the GEMM's where the call goes there
  const size_t a = rows <= GEMV_REG_MAX_ROWS ? gemv_workspace_bytes(w, rows, sms) : 0;
  const size_t b = reg_eligible(w, nullptr, rows) ? 0 : gemm_workspace_bytes(w->n_out, rows, w->k_in, sms);
  return a > b ? a : b;
}

int nf4b_gemm(const nf4b_weight* w, const void* x, void* y, int rows, int epi, const void* operand,
              void* workspace, size_t workspace_bytes, void* stream) {
  return nf4b_gemm_ex(w, x, y, rows, epi, operand, workspace, workspace_bytes, nullptr, stream);
}

int nf4b_gemm_ex(const nf4b_weight* w, const void* x, void* y, int rows, int epi,
                 const void* operand, void* workspace, size_t workspace_bytes,
                 const nf4b_gemm_opts* opts, void* stream) {
  int st = check_weight(w);
  if (st) return st;
  if (x == nullptr || y == nullptr) return fail(NF4B_ERR_ARG, "x or y is null");
  if (rows <= 0) return fail(NF4B_ERR_SHAPE, "rows must be positive (got %d)", rows);
  if (epi < NF4B_EPI_NONE || epi > NF4B_EPI_SILU_GATE) return fail(NF4B_ERR_ARG, "unknown epilogue %d", epi);
  if (epi != NF4B_EPI_NONE && operand == nullptr)
    return fail(NF4B_ERR_ARG, "epilogue %d needs an operand", epi);
  if (!aligned(x, 16)) return fail(NF4B_ERR_ALIGN, "x is not 16-byte aligned");
  if (!aligned(y, 2) || (operand && !aligned(operand, 2)))
    return fail(NF4B_ERR_ALIGN, "y/operand not 2-byte aligned");
  bool f16 = false;
  if ((st = act_type(opts, &f16))) return st;
  if ((st = check_device())) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);

  // The register-fed GEMV for 1..8 rows where it applies; otherwise bf16
  // 1..8 rows on the TMA-ring pair kernel or the block kernel, and every other
  // call (9+ rows, or fp16 outside the register-fed kernel's envelope: the
  // other GEMV kernels are bf16 only) on the tcgen05 GEMM, which from 9 rows
  // on beats the block kernel (2560x9728 at M = 32: 99 against 181 us per
  // layer of five projections).
  if (reg_eligible(w, nullptr, rows) || (!f16 && rows <= GEMV_REG_MAX_ROWS))
    return gemv_call(w, nullptr, x, y, rows, epi, operand, workspace, workspace_bytes, opts, s);
  if (opts != nullptr && opts->norm_weight != nullptr)
    return fail(NF4B_ERR_SHAPE, "a fused RMSNorm is served by the decode GEMV only (got %d rows)", rows);

  GemmParams p = {};
  p.packed = w->packed;
  p.a8 = w->absmax_code;
  p.absmax = w->absmax;
  p.code2 = w->code2;
  p.offset = w->offset;
  p.N = w->n_out;
  p.K = w->k_in;
  p.nested = w->nested ? 1 : 0;
  p.bs_shift = log2i(w->blocksize);
  p.bs2_shift = w->nested ? log2i(w->blocksize2) : 0;
  p.x = static_cast<const uint16_t*>(x);
  p.y = static_cast<uint16_t*>(y);
  p.operand = static_cast<const uint16_t*>(operand);
  p.M = rows;
  p.epi = epi;
  p.f16 = f16 ? 1 : 0;
  // split-K when the caller's workspace holds the partial sums (else one pass)
  const int sms = current_sm_count();
  p.bt = gemm_bt(w->n_out, rows, w->k_in, sms);
  int splits = gemm_splits(w->n_out, rows, w->k_in, sms);
  const size_t need = splits > 1 ? GEMM_COUNTER_BYTES + (size_t)splits * rows * w->n_out * sizeof(float) : 0;
  if (splits > 1 && (workspace == nullptr || workspace_bytes < need || !aligned(workspace, 256))) splits = 1;
  p.splits = splits;
  p.counters = static_cast<int*>(workspace);
  p.partial = splits > 1 ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + GEMM_COUNTER_BYTES) : nullptr;
  return launch_status(launch_gemm_tc(p, s), "nf4 tcgen05 gemm launch");
}

extern "C" int nf4b_gemm_qkv_rope(const nf4b_weight* w, const void* x, void* y, const nf4b_rope_kv* rk,
                                  void* workspace, size_t workspace_bytes, const nf4b_gemm_opts* opts, void* stream) {
  int st = check_weight(w);
  if (st) return st;
  if (x == nullptr || y == nullptr || rk == nullptr) return fail(NF4B_ERR_ARG, "x, y or the rotary store is null");
  if (rk->freqs == nullptr || rk->pos == nullptr || rk->q_out == nullptr || rk->k_cache == nullptr ||
      rk->v_cache == nullptr)
    return fail(NF4B_ERR_ARG, "a rotary store pointer is null");
  if (rk->freqs_dtype < NF4B_F32 || rk->freqs_dtype > NF4B_BF16)
    return fail(NF4B_ERR_DTYPE, "unknown rotary table dtype %d", rk->freqs_dtype);
  if (rk->n_head <= 0 || rk->n_kv <= 0 || rk->n_head % rk->n_kv || rk->max_len <= 0 ||
      (long long)(rk->n_head + 2 * rk->n_kv) * 128 != w->n_out)
    return fail(NF4B_ERR_SHAPE, "n_out %d is not (%d + 2 x %d) heads of 128", w->n_out, rk->n_head, rk->n_kv);
  if (!aligned(x, 16)) return fail(NF4B_ERR_ALIGN, "x is not 16-byte aligned");
  if (!aligned(y, 2) || !aligned(rk->q_out, 2) || !aligned(rk->k_cache, 2) || !aligned(rk->v_cache, 2) ||
      !i64_aligned(rk->pos) || !freqs_aligned(rk->freqs, rk->freqs_dtype))
    return fail(NF4B_ERR_ALIGN, "y/q/cache not 2-byte aligned, pos not 8-byte aligned or freqs misaligned");
  if ((st = check_device())) return st;
  return gemv_call(w, nullptr, x, y, 1, NF4B_EPI_NONE, nullptr, workspace, workspace_bytes, opts,
                   reinterpret_cast<cudaStream_t>(stream), rk);
}

int nf4b_gemm_gated(const nf4b_weight* w1, const nf4b_weight* w3, const void* x, void* y, int rows,
                    void* workspace, size_t workspace_bytes, const nf4b_gemm_opts* opts, void* stream) {
  int st = check_weight(w1);
  if (st) return st;
  if ((st = check_weight(w3))) return st;
  if (w3->n_out != w1->n_out || w3->k_in != w1->k_in || w3->blocksize != w1->blocksize ||
      w3->nested != w1->nested || (w1->nested && w3->blocksize2 != w1->blocksize2))
    return fail(NF4B_ERR_SHAPE, "w1 and w3 differ in shape or quantisation");
  if (x == nullptr || y == nullptr) return fail(NF4B_ERR_ARG, "x or y is null");
  if (rows <= 0) return fail(NF4B_ERR_SHAPE, "rows must be positive (got %d)", rows);
  if (!aligned(x, 16)) return fail(NF4B_ERR_ALIGN, "x is not 16-byte aligned");
  if (!aligned(y, 2)) return fail(NF4B_ERR_ALIGN, "y is not 2-byte aligned");
  if ((st = check_device())) return st;
  return gemv_call(w1, w3, x, y, rows, NF4B_EPI_NONE, nullptr, workspace, workspace_bytes, opts,
                   reinterpret_cast<cudaStream_t>(stream));
}

namespace {

// Validate a chain and fill the kernel parameters (pointers, maps, plan).
int build_chain(const nf4b_chain_job* jobs, int n_jobs, int rows, ChainParams* cp, size_t* partial_bytes) {
  if (jobs == nullptr || n_jobs <= 0) return fail(NF4B_ERR_ARG, "empty job list");
  if (n_jobs > CHAIN_MAX_JOBS)
    return fail(NF4B_ERR_SHAPE, "%d jobs exceed the chain limit of %d", n_jobs, CHAIN_MAX_JOBS);
  if (rows < 1 || rows > 4) return fail(NF4B_ERR_SHAPE, "the GEMV chain serves 1..4 rows (got %d)", rows);
  cp->n_jobs = n_jobs;
  cp->M = rows;
  // The register-fed chain (as the separate calls it must equal) serves rows
  // <= 2 when every job's packed weights are 32-byte aligned.
  cp->reg = rows <= 2 ? 1 : 0;
  for (int i = 0; i < n_jobs; ++i) {
    const nf4b_chain_job& jb = jobs[i];
    int st = check_weight(jb.w);
    if (st) return st;
    const nf4b_weight* w = jb.w;
    if (w->blocksize != 64 || w->k_in % 256)
      return fail(NF4B_ERR_SHAPE, "job %d: the chain needs blocksize 64 and k_in %% 256 == 0", i);
    if ((long long)rows * w->k_in * 2 > GEMV_PAIR_X_MAX)
      return fail(NF4B_ERR_SHAPE, "job %d: %d rows x k_in %d do not fit the staged x", i, rows, w->k_in);
    if ((long long)(w->n_out + 15) / 16 > CHAIN_MAX_TILES) return fail(NF4B_ERR_SHAPE, "job %d too large", i);
    if (!use_pairs(w, rows)) return fail(NF4B_ERR_ALIGN, "job %d: scales not aligned for the copies", i);
    if (jb.x == nullptr || jb.y == nullptr) return fail(NF4B_ERR_ARG, "job %d: x or y is null", i);
    if (!aligned(jb.x, 16)) return fail(NF4B_ERR_ALIGN, "job %d: x is not 16-byte aligned", i);
    if (!aligned(jb.y, 2) || (jb.operand && !aligned(jb.operand, 2)) || (jb.norm_weight && !aligned(jb.norm_weight, 2)))
      return fail(NF4B_ERR_ALIGN, "job %d: y/operand/norm weight not 2-byte aligned", i);
    if (jb.norm_weight != nullptr && !(jb.norm_eps >= 0.f))
      return fail(NF4B_ERR_ARG, "job %d: norm eps must be >= 0", i);
    ChainJob& J = cp->jobs[i];
    J.gated = jb.w3 != nullptr ? 1 : 0;
    if (J.gated) {
      const nf4b_weight* w3 = jb.w3;
      if ((st = check_weight(w3))) return st;
      if (w3->n_out != w->n_out || w3->k_in != w->k_in || w3->blocksize != w->blocksize ||
          w3->nested != w->nested || (w->nested && w3->blocksize2 != w->blocksize2) || !use_pairs(w3, rows))
        return fail(NF4B_ERR_SHAPE, "job %d: the gated pair's weights differ in shape or quantisation", i);
    } else {
      if (jb.epi < NF4B_EPI_NONE || jb.epi > NF4B_EPI_SILU_GATE)
        return fail(NF4B_ERR_ARG, "job %d: unknown epilogue %d", i, jb.epi);
      if (jb.epi != NF4B_EPI_NONE && jb.operand == nullptr)
        return fail(NF4B_ERR_ARG, "job %d: epilogue %d needs an operand", i, jb.epi);
    }
    const uint64_t rb = (uint64_t)w->k_in / 2;
    if (!make_map_2d(&J.wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->packed, rb, (uint64_t)w->n_out, rb, 128, 16,
                     CU_TENSOR_MAP_SWIZZLE_NONE) ||
        (J.gated && !make_map_2d(&J.wmap3, CU_TENSOR_MAP_DATA_TYPE_UINT8, jb.w3->packed, rb, (uint64_t)w->n_out,
                                 rb, 128, 16, CU_TENSOR_MAP_SWIZZLE_NONE)))
      return fail(NF4B_ERR_ARG, "job %d: cannot describe the weight to the TMA unit", i);
    J.packed = w->packed;
    J.packed3 = J.gated ? jb.w3->packed : nullptr;
    if (!aligned(w->packed, 32) || (J.gated && !aligned(jb.w3->packed, 32)) ||
        (long long)w->n_out * (w->k_in / 64) >= (1LL << 31))
      cp->reg = 0;
    J.a8 = w->absmax_code;
    J.absmax = w->absmax;
    J.code2 = w->code2;
    J.offset = w->offset;
    J.a8_3 = J.gated ? jb.w3->absmax_code : nullptr;
    J.absmax3 = J.gated ? jb.w3->absmax : nullptr;
    J.code2_3 = J.gated ? jb.w3->code2 : nullptr;
    J.offset3 = J.gated ? jb.w3->offset : 0.f;
    J.x = static_cast<const uint16_t*>(jb.x);
    J.y = static_cast<uint16_t*>(jb.y);
    J.operand = static_cast<const uint16_t*>(jb.operand);
    J.norm_w = static_cast<const uint16_t*>(jb.norm_weight);
    J.norm_eps = jb.norm_eps;
    J.N = w->n_out;
    J.K = w->k_in;
    J.nested = w->nested ? 1 : 0;
    J.bs2_shift = w->nested ? log2i(w->blocksize2) : 0;
    J.epi = J.gated ? NF4B_EPI_NONE : jb.epi;
  }
  *partial_bytes = chain_plan(cp, current_sm_count());
  return NF4B_OK;
}

}  // namespace

extern "C" size_t nf4b_gemv_chain_workspace_size(const nf4b_chain_job* jobs, int n_jobs, int rows) {
  static thread_local ChainParams cp;
  size_t partial = 0;
  if (build_chain(jobs, n_jobs, rows, &cp, &partial)) return 0;
  return GEMV_COUNTER_BYTES + partial;
}

extern "C" int nf4b_gemv_chain(const nf4b_chain_job* jobs, int n_jobs, int rows, void* workspace,
                               size_t workspace_bytes, void* stream) {
  static thread_local ChainParams cp;
  size_t partial = 0;
  int st = build_chain(jobs, n_jobs, rows, &cp, &partial);
  if (st) return st;
  const size_t need = GEMV_COUNTER_BYTES + partial;
  if (workspace == nullptr || workspace_bytes < need)
    return fail(NF4B_ERR_WORKSPACE, "chain workspace of %zu bytes needed, %zu given", need,
                workspace ? workspace_bytes : (size_t)0);
  if (!aligned(workspace, 256)) return fail(NF4B_ERR_ALIGN, "workspace is not 256-byte aligned");
  if ((st = check_device())) return st;
  cp.counters = static_cast<int*>(workspace);
  cp.partial = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + GEMV_COUNTER_BYTES);
  return launch_status(launch_gemv_chain(cp, reinterpret_cast<cudaStream_t>(stream)), "nf4 gemv chain launch");
}

namespace {

// Validate a decode step and fill the kernel parameters.
int build_step(const nf4b_chain_job* jobs, int n_jobs, int rows, StepParams* sp, size_t* bytes) {
  if (jobs == nullptr || n_jobs <= 0) return fail(NF4B_ERR_ARG, "empty job list");
  if (n_jobs > STEP_MAX_JOBS)
    return fail(NF4B_ERR_SHAPE, "%d jobs exceed the decode step limit of %d", n_jobs, STEP_MAX_JOBS);
  if (rows < 1 || rows > 2) return fail(NF4B_ERR_SHAPE, "the decode step serves 1 or 2 rows (got %d)", rows);
  sp->n_jobs = n_jobs;
  sp->M = rows;
  sp->stall_job = -1;
  sp->wait_ns = 2000000000ull;
  for (int i = 0; i < n_jobs; ++i) {
    const nf4b_chain_job& jb = jobs[i];
    int st = check_weight(jb.w);
    if (st) return st;
    const nf4b_weight* w = jb.w;
    if (w->blocksize != 64 || w->k_in % 256 || w->k_in > STEP_MAX_K || w->n_out % 16)
      return fail(NF4B_ERR_SHAPE,
                  "job %d: the decode step needs blocksize 64, k_in %% 256 == 0, k_in <= %d, n_out %% 16 == 0", i,
                  STEP_MAX_K);
    if ((long long)w->n_out * (w->k_in / 64) >= (1LL << 31)) return fail(NF4B_ERR_SHAPE, "job %d too large", i);
    if (!aligned(w->packed, 32) || !use_pairs(w, rows))
      return fail(NF4B_ERR_ALIGN, "job %d: packed weight not 32-byte aligned or scales not aligned", i);
    if (jb.x == nullptr || jb.y == nullptr) return fail(NF4B_ERR_ARG, "job %d: x or y is null", i);
    if (!aligned(jb.x, 16)) return fail(NF4B_ERR_ALIGN, "job %d: x is not 16-byte aligned", i);
    if (!aligned(jb.y, 4) || (jb.operand && !aligned(jb.operand, 2)) || (jb.norm_weight && !aligned(jb.norm_weight, 16)))
      return fail(NF4B_ERR_ALIGN, "job %d: y not 4-byte, operand not 2-byte or norm weight not 16-byte aligned", i);
    if (jb.norm_weight != nullptr && !(jb.norm_eps >= 0.f))
      return fail(NF4B_ERR_ARG, "job %d: norm eps must be >= 0", i);
    StepJob& J = sp->jobs[i];
    J = StepJob{};
    J.gated = jb.w3 != nullptr ? 1 : 0;
    if (J.gated) {
      const nf4b_weight* w3 = jb.w3;
      if ((st = check_weight(w3))) return st;
      if (w3->n_out != w->n_out || w3->k_in != w->k_in || w3->blocksize != w->blocksize ||
          w3->nested != w->nested || (w->nested && w3->blocksize2 != w->blocksize2) || !use_pairs(w3, rows) ||
          !aligned(w3->packed, 32))
        return fail(NF4B_ERR_SHAPE, "job %d: the gated pair's weights differ in shape, quantisation or alignment", i);
    } else {
      if (jb.epi < NF4B_EPI_NONE || jb.epi > NF4B_EPI_SILU_GATE)
        return fail(NF4B_ERR_ARG, "job %d: unknown epilogue %d", i, jb.epi);
      if (jb.epi != NF4B_EPI_NONE && jb.operand == nullptr)
        return fail(NF4B_ERR_ARG, "job %d: epilogue %d needs an operand", i, jb.epi);
    }
    if (i > 0) {
      const nf4b_chain_job& pv = jobs[i - 1];
      if (jb.x == pv.y && w->k_in != pv.w->n_out)
        return fail(NF4B_ERR_SHAPE, "job %d: x is job %d's y but k_in %d != its n_out %d", i, i - 1, w->k_in,
                    pv.w->n_out);
      if (jb.operand != nullptr && jb.operand == pv.y && w->n_out != pv.w->n_out)
        return fail(NF4B_ERR_SHAPE, "job %d: the operand is job %d's y of another width", i, i - 1);
    }
    J.packed = w->packed;
    J.a8 = w->absmax_code;
    J.absmax = w->absmax;
    J.code2 = w->code2;
    J.offset = w->offset;
    J.packed3 = J.gated ? jb.w3->packed : nullptr;
    J.a8_3 = J.gated ? jb.w3->absmax_code : nullptr;
    J.absmax3 = J.gated ? jb.w3->absmax : nullptr;
    J.code2_3 = J.gated ? jb.w3->code2 : nullptr;
    J.offset3 = J.gated ? jb.w3->offset : 0.f;
    J.x = static_cast<const uint16_t*>(jb.x);
    J.y = static_cast<uint16_t*>(jb.y);
    J.operand = static_cast<const uint16_t*>(jb.operand);
    J.norm_w = static_cast<const uint16_t*>(jb.norm_weight);
    J.norm_eps = jb.norm_eps;
    J.N = w->n_out;
    J.K = w->k_in;
    J.nested = w->nested ? 1 : 0;
    J.bs2_shift = w->nested ? log2i(w->blocksize2) : 0;
    J.epi = J.gated ? NF4B_EPI_NONE : jb.epi;
  }
  *bytes = step_plan(sp, current_sm_count());
  return NF4B_OK;
}

int decode_step_call(const nf4b_chain_job* jobs, int n_jobs, int rows, void* workspace, size_t workspace_bytes,
                     int stall_job, unsigned long long wait_ns, void* stream) {
  static thread_local StepParams sp;
  size_t need = 0;
  int st = build_step(jobs, n_jobs, rows, &sp, &need);
  if (st) return st;
  if (workspace == nullptr || workspace_bytes < need)
    return fail(NF4B_ERR_WORKSPACE, "decode step workspace of %zu bytes needed, %zu given", need,
                workspace ? workspace_bytes : (size_t)0);
  if (!aligned(workspace, 256)) return fail(NF4B_ERR_ALIGN, "workspace is not 256-byte aligned");
  if ((st = check_device())) return st;
  sp.stall_job = stall_job;
  sp.wait_ns = wait_ns;
  return launch_status(launch_decode_step(sp, workspace, reinterpret_cast<cudaStream_t>(stream)),
                       "nf4 decode step launch");
}

}  // namespace

extern "C" size_t nf4b_decode_step_workspace_size(const nf4b_chain_job* jobs, int n_jobs, int rows) {
  static thread_local StepParams sp;
  size_t need = 0;
  if (build_step(jobs, n_jobs, rows, &sp, &need)) return 0;
  return need;
}

extern "C" int nf4b_decode_step(const nf4b_chain_job* jobs, int n_jobs, int rows, void* workspace,
                                size_t workspace_bytes, void* stream) {
  return decode_step_call(jobs, n_jobs, rows, workspace, workspace_bytes, -1, 2000000000ull, stream);
}

extern "C" int nf4b_debug_decode_step(const nf4b_chain_job* jobs, int n_jobs, int rows, void* workspace,
                                      size_t workspace_bytes, int stall_job, unsigned long long wait_ns,
                                      void* stream) {
  if (wait_ns == 0 || wait_ns > 2000000000ull) return fail(NF4B_ERR_ARG, "wait_ns must be in (0, 2e9]");
  return decode_step_call(jobs, n_jobs, rows, workspace, workspace_bytes, stall_job, wait_ns, stream);
}

extern "C" int nf4b_debug_gemm_hook(int skip_x0, unsigned long long wait_ns) {
  if (wait_ns == 0 || wait_ns > 2000000000ull) return fail(NF4B_ERR_ARG, "wait_ns must be in (0, 2e9]");
  if (skip_x0 != 0 && skip_x0 != 1) return fail(NF4B_ERR_ARG, "skip_x0 must be 0 or 1");
  int st = check_device();
  if (st) return st;
  return set_gemm_debug(skip_x0, wait_ns) == 0 ? 0 : fail(NF4B_ERR_LAUNCH, "setting the GEMM test hook failed");
}

extern "C" int nf4b_dense_gemv(const void* w, const void* x, void* y, int n_out, int k_in, const void* norm_weight,
                               float norm_eps, void* stream) {
  if (w == nullptr || x == nullptr || y == nullptr) return fail(NF4B_ERR_ARG, "null pointer");
  if (norm_weight != nullptr && (!aligned(norm_weight, 2) || !(norm_eps >= 0.f)))
    return fail(NF4B_ERR_ARG, "norm weight not 2-byte aligned or eps < 0");
  if (n_out <= 0) return fail(NF4B_ERR_SHAPE, "n_out must be positive (got %d)", n_out);
  if (k_in != 1024 && k_in != 2048 && k_in != 2560 && k_in != 4096)
    return fail(NF4B_ERR_SHAPE, "k_in %d is not one of 1024, 2048, 2560, 4096", k_in);
  if (!aligned(w, 16) || !aligned(x, 16) || !aligned(y, 2)) return fail(NF4B_ERR_ALIGN, "w/x not 16-byte aligned");
  int st = check_device();
  if (st) return st;
  return launch_status(launch_dense_gemv(static_cast<const uint16_t*>(w), static_cast<const uint16_t*>(x),
                                         static_cast<uint16_t*>(y), n_out, k_in, current_sm_count(),
                                         static_cast<const uint16_t*>(norm_weight), norm_eps,
                                         reinterpret_cast<cudaStream_t>(stream)),
                       "dense gemv launch");
}

extern "C" size_t nf4b_sample_workspace_size(int vocab) {
  if (vocab <= 0 || vocab > SAMPLER_MAX_VOCAB) return 0;
  return sampler_workspace_bytes(vocab);
}

extern "C" int nf4b_sample(const void* logits, int vocab, float temperature, float top_p, int top_k,
                           unsigned long long seed, const int64_t* step, int64_t* out, void* workspace,
                           size_t workspace_bytes, void* stream) {
  if (logits == nullptr || out == nullptr) return fail(NF4B_ERR_ARG, "null pointer");
  if (vocab <= 0 || vocab > SAMPLER_MAX_VOCAB)
    return fail(NF4B_ERR_SHAPE, "vocabulary %d outside [1, %d]", vocab, SAMPLER_MAX_VOCAB);
  if (!(temperature >= 0.f) || !(top_p >= 0.f) || top_k < 1)
    return fail(NF4B_ERR_ARG, "bad sampling parameters (temperature %g, top_p %g, top_k %d)", temperature, top_p,
                top_k);
  const size_t need = sampler_workspace_bytes(vocab);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(NF4B_ERR_WORKSPACE, "sampler workspace of %zu bytes needed, %zu given", need,
                workspace ? workspace_bytes : (size_t)0);
  if (!aligned(workspace, 256) || !aligned(logits, 2) || !i64_aligned(out) || !i64_aligned(step))
    return fail(NF4B_ERR_ALIGN, "workspace/logits/out/step misaligned");
  int st = check_device();
  if (st) return st;
  return launch_status(launch_sampler(static_cast<const uint16_t*>(logits), vocab, temperature, top_p, top_k, seed,
                                      step, out, workspace, reinterpret_cast<cudaStream_t>(stream)),
                       "sampler launch");
}

extern "C" int nf4b_embed_rows(const void* table, long long rows, const int64_t* ids, int n_ids, int dim, void* out,
                               void* stream) {
  if (table == nullptr || ids == nullptr || out == nullptr) return fail(NF4B_ERR_ARG, "null pointer");
  if (rows <= 0 || n_ids <= 0 || dim <= 0 || dim % 8)
    return fail(NF4B_ERR_SHAPE, "embedding of %lld rows, %d ids, dim %d (dim %% 8 == 0)", rows, n_ids, dim);
  if (!aligned(table, 16) || !aligned(out, 16) || !aligned(ids, 8))
    return fail(NF4B_ERR_ALIGN, "table/out not 16-byte aligned or ids not 8-byte aligned");
  int st = check_device();
  if (st) return st;
  return launch_status(launch_embed_rows(static_cast<const uint16_t*>(table), rows, ids, n_ids, dim,
                                         static_cast<uint16_t*>(out), reinterpret_cast<cudaStream_t>(stream)),
                       "embedding gather launch");
}

extern "C" int nf4b_frame_select(const int64_t* main_tok, const int64_t* high_tok, const int64_t* recent,
                                 int n_recent, long long sem_begin, long long codebook_size, int64_t* tokens,
                                 const void* fast_emb, int dim, void* h, void* stream) {
  if (main_tok == nullptr || high_tok == nullptr || tokens == nullptr || fast_emb == nullptr || h == nullptr ||
      (n_recent > 0 && recent == nullptr))
    return fail(NF4B_ERR_ARG, "null pointer");
  if (n_recent < 0 || codebook_size <= 0 || dim <= 0 || dim % 8)
    return fail(NF4B_ERR_SHAPE, "recent window %d, codebook size %lld, dim %d (dim %% 8 == 0)", n_recent,
                codebook_size, dim);
  if (!aligned(fast_emb, 16) || !aligned(h, 16)) return fail(NF4B_ERR_ALIGN, "fast_emb/h not 16-byte aligned");
  if (!i64_aligned(main_tok) || !i64_aligned(high_tok) || !i64_aligned(recent) || !i64_aligned(tokens))
    return fail(NF4B_ERR_ALIGN, "token ids not 8-byte aligned");
  int st = check_device();
  if (st) return st;
  return launch_status(launch_frame_select(main_tok, high_tok, recent, n_recent, sem_begin, codebook_size, tokens,
                                           static_cast<const uint16_t*>(fast_emb), dim, static_cast<uint16_t*>(h),
                                           reinterpret_cast<cudaStream_t>(stream)),
                       "frame select launch");
}

extern "C" int nf4b_frame_advance(const void* sem_emb, long long vocab, const void* cb_emb, long long codebook_size,
                                  int n_codebooks, const int64_t* tokens, int dim, void* x, int64_t* recent,
                                  int n_recent, int64_t* pos, int64_t* step, void* stream) {
  if (sem_emb == nullptr || cb_emb == nullptr || tokens == nullptr || x == nullptr || pos == nullptr ||
      step == nullptr || (n_recent > 0 && recent == nullptr))
    return fail(NF4B_ERR_ARG, "null pointer");
  if (vocab <= 0 || codebook_size <= 0 || n_codebooks < 0 || n_codebooks > FRAME_MAX_CODEBOOKS || dim <= 0 ||
      n_recent < 0)
    return fail(NF4B_ERR_SHAPE, "vocab %lld, codebooks %d x %lld, dim %d, recent %d", vocab, n_codebooks,
                codebook_size, dim, n_recent);
  if (!aligned(sem_emb, 2) || !aligned(cb_emb, 2) || !aligned(x, 2)) return fail(NF4B_ERR_ALIGN, "bf16 misaligned");
  if (!i64_aligned(tokens) || !i64_aligned(recent) || !i64_aligned(pos) || !i64_aligned(step))
    return fail(NF4B_ERR_ALIGN, "tokens/recent/pos/step not 8-byte aligned");
  int st = check_device();
  if (st) return st;
  return launch_status(launch_frame_advance(static_cast<const uint16_t*>(sem_emb), vocab,
                                            static_cast<const uint16_t*>(cb_emb), codebook_size, n_codebooks, tokens,
                                            dim, static_cast<uint16_t*>(x), recent, n_recent, pos, step,
                                            reinterpret_cast<cudaStream_t>(stream)),
                       "frame advance launch");
}

extern "C" int nf4b_dequantize(const nf4b_weight* w, void* out, void* stream) {
  int st = check_weight(w);
  if (st) return st;
  if (out == nullptr) return fail(NF4B_ERR_ARG, "out is null");
  if (!aligned(out, 16)) return fail(NF4B_ERR_ALIGN, "out is not 16-byte aligned");
  if ((st = check_device())) return st;
  DequantParams p;
  p.packed = w->packed;
  p.a8 = w->absmax_code;
  p.absmax = w->absmax;
  p.code2 = w->code2;
  p.offset = w->offset;
  p.N = w->n_out;
  p.K = w->k_in;
  p.nested = w->nested ? 1 : 0;
  p.bs_shift = log2i(w->blocksize);
  p.bs2_shift = w->nested ? log2i(w->blocksize2) : 0;
  p.out = static_cast<uint16_t*>(out);
  return launch_status(launch_dequant(p, reinterpret_cast<cudaStream_t>(stream)), "nf4 dequantize launch");
}

}  // extern "C"

namespace {
// The activation type argument of the elementwise _ex calls: NF4B_BF16 or NF4B_F16.
int elem_type(int dtype, bool* f16) {
  *f16 = dtype == NF4B_F16;
  if (dtype != NF4B_BF16 && dtype != NF4B_F16)
    return fail(NF4B_ERR_DTYPE, "activation dtype %d is not served (NF4B_BF16 or NF4B_F16)", dtype);
  return NF4B_OK;
}
}  // namespace

extern "C" {

int nf4b_rms_norm(const void* x, const void* weight, void* y, int rows, int width, float eps, void* stream) {
  return nf4b_rms_norm_ex(x, weight, y, rows, width, eps, NF4B_BF16, stream);
}

int nf4b_rms_norm_ex(const void* x, const void* weight, void* y, int rows, int width, float eps, int dtype,
                     void* stream) {
  bool f16 = false;
  if (int e = elem_type(dtype, &f16)) return e;
  if (x == nullptr || weight == nullptr || y == nullptr) return fail(NF4B_ERR_ARG, "null pointer");
  if (rows <= 0 || width <= 0) return fail(NF4B_ERR_SHAPE, "empty input %dx%d", rows, width);
  if (!(eps >= 0.f)) return fail(NF4B_ERR_ARG, "eps must be >= 0");
  if (!aligned(x, 2) || !aligned(weight, 2) || !aligned(y, 2))
    return fail(NF4B_ERR_ALIGN, "x/weight/y not 2-byte aligned");
  int st = check_device();
  if (st) return st;
  return launch_status(
      launch_rms_norm(static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(weight),
                      static_cast<uint16_t*>(y), rows, width, eps,
                      reinterpret_cast<cudaStream_t>(stream), f16),
      "rms_norm launch");
}

int nf4b_rope(const void* x, const void* freqs, int freqs_dtype, void* y, int batch, int seq,
              int heads, int head_dim, void* stream) {
  return nf4b_rope_ex(x, freqs, freqs_dtype, y, batch, seq, heads, head_dim, NF4B_BF16, stream);
}

int nf4b_rope_ex(const void* x, const void* freqs, int freqs_dtype, void* y, int batch, int seq,
                 int heads, int head_dim, int dtype, void* stream) {
  bool f16 = false;
  if (int e = elem_type(dtype, &f16)) return e;
  if (x == nullptr || freqs == nullptr || y == nullptr) return fail(NF4B_ERR_ARG, "null pointer");
  if (batch <= 0 || seq <= 0 || heads <= 0 || head_dim <= 0 || head_dim % 2)
    return fail(NF4B_ERR_SHAPE, "bad rotary shape (%d,%d,%d,%d)", batch, seq, heads, head_dim);
  if (freqs_dtype < NF4B_F32 || freqs_dtype > NF4B_BF16)
    return fail(NF4B_ERR_DTYPE, "unknown freqs dtype %d", freqs_dtype);
  if (!aligned(x, 2) || !aligned(y, 2) || !freqs_aligned(freqs, freqs_dtype))
    return fail(NF4B_ERR_ALIGN, "x/y not 2-byte aligned or freqs misaligned");
  int st = check_device();
  if (st) return st;
  const long long pairs = (long long)batch * seq * heads * head_dim / 2;
  return launch_status(launch_rope(static_cast<const uint16_t*>(x), freqs, freqs_dtype,
                                   static_cast<uint16_t*>(y), pairs, head_dim / 2, heads, seq,
                                   reinterpret_cast<cudaStream_t>(stream), f16),
                       "rope launch");
}

int nf4b_qk_rope_kv(const void* qkv, const void* q_norm_w, const void* k_norm_w, float eps,
                    const void* freqs, int freqs_dtype, const int64_t* pos, void* q_out,
                    void* k_cache, void* v_cache, int n_head, int n_kv, int head_dim, int max_len,
                    void* stream) {
  return nf4b_qk_rope_kv_ex(qkv, q_norm_w, k_norm_w, eps, freqs, freqs_dtype, pos, q_out, k_cache, v_cache, n_head,
                            n_kv, head_dim, max_len, NF4B_BF16, stream);
}

int nf4b_qk_rope_kv_ex(const void* qkv, const void* q_norm_w, const void* k_norm_w, float eps,
                       const void* freqs, int freqs_dtype, const int64_t* pos, void* q_out,
                       void* k_cache, void* v_cache, int n_head, int n_kv, int head_dim, int max_len,
                       int dtype, void* stream) {
  bool f16 = false;
  if (int e = elem_type(dtype, &f16)) return e;
  if (!qkv || !freqs || !pos || !q_out || !k_cache || !v_cache)
    return fail(NF4B_ERR_ARG, "null pointer");
  if (head_dim != 128) return fail(NF4B_ERR_SHAPE, "head_dim must be 128 (got %d)", head_dim);
  if (n_head <= 0 || n_kv <= 0 || max_len <= 0) return fail(NF4B_ERR_SHAPE, "bad head counts");
  if ((q_norm_w == nullptr) != (k_norm_w == nullptr))
    return fail(NF4B_ERR_ARG, "q and k norm weights must both be given or both be null");
  if (freqs_dtype < NF4B_F32 || freqs_dtype > NF4B_BF16)
    return fail(NF4B_ERR_DTYPE, "unknown freqs dtype %d", freqs_dtype);
  if (!aligned(qkv, 2) || !aligned(q_norm_w, 2) || !aligned(k_norm_w, 2) || !aligned(q_out, 2) ||
      !aligned(k_cache, 2) || !aligned(v_cache, 2) || !i64_aligned(pos) || !freqs_aligned(freqs, freqs_dtype))
    return fail(NF4B_ERR_ALIGN, "activations/caches not 2-byte aligned, pos not 8-byte aligned or freqs misaligned");
  int st = check_device();
  if (st) return st;
  return launch_status(
      launch_qk_rope_kv(static_cast<const uint16_t*>(qkv), static_cast<const uint16_t*>(q_norm_w),
                        static_cast<const uint16_t*>(k_norm_w), eps, freqs, freqs_dtype, pos,
                        static_cast<uint16_t*>(q_out), static_cast<uint16_t*>(k_cache),
                        static_cast<uint16_t*>(v_cache), n_head, n_kv, max_len,
                        reinterpret_cast<cudaStream_t>(stream), f16),
      "qk_rope_kv launch");
}

size_t nf4b_decode_attention_workspace_size(int n_head, int head_dim, int window) {
  if (n_head <= 0 || head_dim <= 0 || window <= 0) return 0;
  AttnPlan plan;
  attn_plan(n_head, head_dim, window, &plan);
  return plan.counter_bytes + plan.partial_bytes;
}

int nf4b_decode_attention(const void* q, const void* k_cache, const void* v_cache,
                          const int64_t* pos, const uint8_t* mask, void* out, int n_head, int n_kv,
                          int head_dim, int max_len, int window, void* workspace,
                          size_t workspace_bytes, void* stream) {
  return nf4b_decode_attention_ex(q, k_cache, v_cache, pos, mask, out, n_head, n_kv, head_dim, max_len, window,
                                  workspace, workspace_bytes, NF4B_BF16, stream);
}

int nf4b_decode_attention_ex(const void* q, const void* k_cache, const void* v_cache,
                             const int64_t* pos, const uint8_t* mask, void* out, int n_head, int n_kv,
                             int head_dim, int max_len, int window, void* workspace,
                             size_t workspace_bytes, int dtype, void* stream) {
  bool f16 = false;
  if (int e = elem_type(dtype, &f16)) return e;
  if (!q || !k_cache || !v_cache || !out) return fail(NF4B_ERR_ARG, "null pointer");
  if (head_dim != 128) return fail(NF4B_ERR_SHAPE, "head_dim must be 128 (got %d)", head_dim);
  if (n_head <= 0 || n_kv <= 0 || n_head % n_kv)
    return fail(NF4B_ERR_SHAPE, "n_head %d is not a multiple of n_kv %d", n_head, n_kv);
  if ((size_t)n_kv * sizeof(int) > ATTN_COUNTER_BYTES)
    return fail(NF4B_ERR_SHAPE, "more than %zu KV heads", ATTN_COUNTER_BYTES / sizeof(int));
  const int groups = n_head / n_kv;
  if (groups != 1 && groups != 2 && groups != 4 && groups != 8)
    return fail(NF4B_ERR_SHAPE, "query groups of %d are not served (1, 2, 4 or 8)", groups);
  if (window <= 0 || window > max_len) return fail(NF4B_ERR_SHAPE, "window %d outside [1, %d]", window, max_len);
  if (!aligned(q, 16) || !aligned(k_cache, 16) || !aligned(v_cache, 16))
    return fail(NF4B_ERR_ALIGN, "q / caches not 16-byte aligned");
  if (!aligned(out, 2) || !i64_aligned(pos)) return fail(NF4B_ERR_ALIGN, "out not 2-byte or pos not 8-byte aligned");
  AttnPlan plan;
  attn_plan(n_head, head_dim, window, &plan);
  const size_t need = plan.counter_bytes + plan.partial_bytes;
  if (workspace == nullptr || workspace_bytes < need)
    return fail(NF4B_ERR_WORKSPACE, "workspace of %zu bytes needed", need);
  if (!aligned(workspace, 256)) return fail(NF4B_ERR_ALIGN, "workspace is not 256-byte aligned");
  int st = check_device();
  if (st) return st;
  float* partial = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + plan.counter_bytes);
  return launch_status(
      launch_decode_attention(static_cast<const uint16_t*>(q), static_cast<const uint16_t*>(k_cache),
                              static_cast<const uint16_t*>(v_cache), pos, mask, static_cast<uint16_t*>(out),
                              n_head, n_kv, max_len, window, partial, static_cast<int*>(workspace),
                              reinterpret_cast<cudaStream_t>(stream), f16),
      "decode attention launch");
}

int nf4b_qkv_attention(const void* qkv, const void* q_norm_w, const void* k_norm_w, float eps,
                       const void* freqs, int freqs_dtype, const int64_t* pos, void* q_scratch,
                       void* k_cache, void* v_cache, void* out, int n_head, int n_kv, int head_dim, int max_len,
                       int window, void* workspace, size_t workspace_bytes, void* stream) {
  return nf4b_qkv_attention_ex(qkv, q_norm_w, k_norm_w, eps, freqs, freqs_dtype, pos, q_scratch, k_cache, v_cache,
                               out, n_head, n_kv, head_dim, max_len, window, workspace, workspace_bytes, NF4B_BF16,
                               stream);
}

int nf4b_qkv_attention_ex(const void* qkv, const void* q_norm_w, const void* k_norm_w, float eps,
                          const void* freqs, int freqs_dtype, const int64_t* pos, void* q_scratch,
                          void* k_cache, void* v_cache, void* out, int n_head, int n_kv, int head_dim,
                          int max_len, int window, void* workspace, size_t workspace_bytes, int dtype,
                          void* stream) {
  bool f16 = false;
  if (int e = elem_type(dtype, &f16)) return e;
  if (!qkv || !freqs || !pos || !q_scratch || !k_cache || !v_cache || !out) return fail(NF4B_ERR_ARG, "null pointer");
  if (head_dim != 128) return fail(NF4B_ERR_SHAPE, "head_dim must be 128 (got %d)", head_dim);
  if (n_head <= 0 || n_kv <= 0 || n_head % n_kv)
    return fail(NF4B_ERR_SHAPE, "n_head %d is not a multiple of n_kv %d", n_head, n_kv);
  if ((size_t)n_kv * sizeof(int) > ATTN_COUNTER_BYTES)
    return fail(NF4B_ERR_SHAPE, "more than %zu KV heads", ATTN_COUNTER_BYTES / sizeof(int));
  const int groups = n_head / n_kv;
  if (groups != 1 && groups != 2 && groups != 4 && groups != 8)
    return fail(NF4B_ERR_SHAPE, "query groups of %d are not served (1, 2, 4 or 8)", groups);
  if (window <= 0 || window > max_len) return fail(NF4B_ERR_SHAPE, "window %d outside [1, %d]", window, max_len);
  if ((q_norm_w == nullptr) != (k_norm_w == nullptr))
    return fail(NF4B_ERR_ARG, "q and k norm weights must both be given or both be null");
  if (freqs_dtype < NF4B_F32 || freqs_dtype > NF4B_BF16)
    return fail(NF4B_ERR_DTYPE, "unknown freqs dtype %d", freqs_dtype);
  if (!aligned(q_scratch, 16) || !aligned(k_cache, 16) || !aligned(v_cache, 16))
    return fail(NF4B_ERR_ALIGN, "q scratch / caches not 16-byte aligned");
  if (!aligned(qkv, 2) || !aligned(q_norm_w, 2) || !aligned(k_norm_w, 2) || !aligned(out, 2) || !i64_aligned(pos) ||
      !freqs_aligned(freqs, freqs_dtype))
    return fail(NF4B_ERR_ALIGN, "qkv/norm weights/out not 2-byte aligned, pos not 8-byte aligned or freqs misaligned");
  AttnPlan plan;
  attn_plan(n_head, head_dim, window, &plan);
  const size_t need = plan.counter_bytes + plan.partial_bytes;
  if (workspace == nullptr || workspace_bytes < need)
    return fail(NF4B_ERR_WORKSPACE, "workspace of %zu bytes needed", need);
  if (!aligned(workspace, 256)) return fail(NF4B_ERR_ALIGN, "workspace is not 256-byte aligned");
  int st = check_device();
  if (st) return st;
  QkvIn in;
  in.qkv = static_cast<const uint16_t*>(qkv);
  in.qw = static_cast<const uint16_t*>(q_norm_w);
  in.kw = static_cast<const uint16_t*>(k_norm_w);
  in.eps = eps;
  in.freqs = freqs;
  in.ftype = freqs_dtype;
  in.n_head = n_head;
  float* partial = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + plan.counter_bytes);
  return launch_status(
      launch_qkv_attention(in, pos, static_cast<uint16_t*>(q_scratch), static_cast<uint16_t*>(k_cache),
                           static_cast<uint16_t*>(v_cache), static_cast<uint16_t*>(out), n_head, n_kv, max_len,
                           window, partial, static_cast<int*>(workspace), reinterpret_cast<cudaStream_t>(stream),
                           f16),
      "qkv attention launch");
}

}  // extern "C"
