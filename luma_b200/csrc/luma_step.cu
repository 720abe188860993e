// luma_step.cu — sm_100a kernels and C ABI of the LUMA optimizer step.
//
// The step is the reference's two-pass matched-scaling update
// (IgorYashch/LUMA src/luma_optimizer/functional.py:183-298), run for every
// tensor of the optimizer in two launches over a device descriptor table:
//
//   pass 1  decode (Q_m, Q_w) on the tensor's current grid -> EMA with the
//           gradient -> per-thread max |m'|, max v' -> warp/block reduction ->
//           one atomicMax per (CTA, tensor) on the float bit patterns (order-
//           independent, so deterministic).  The CTA whose octet count closes
//           the tensor (atomic counter, no spinning) turns the two maxima into
//           the next grid in float64 (functional.py:74-92, 282-292).
//   pass 2  decode -> EMA (recomputed: no temporaries) -> AdamW update of the
//           param in place -> LogSR re-quantization on the new grid with
//           Philox4x32-10 uniforms (or injected uniforms, the test hook).
//
// Arithmetic follows the reference op by op as PyTorch's CUDA kernels execute
// it (each op rounds to float32 on its own; a tensor divided by a Python
// scalar s is a multiply by fl32(1.0 / s), the reciprocal taken in float64;
// addcdiv is one fma), so the
// codes and params are bit-identical to the reference running on CUDA when
// both consume the same uniforms.  No fast-math: expm1f, expf, log1pf, logf
// are the CUDA library's accurate versions, the same functions PyTorch's
// element-wise kernels call; division, reciprocal and square root are the
// IEEE intrinsics, or in the steady pass-2 loop branch-free correctly rounded
// forms that equal them on the operand ranges where they are used.
//
// Work split: the flat space of all tensors, counted in octets (8 elements),
// is cut into one contiguous range per CTA of a persistent grid sized from the
// occupancy calculator.  A CTA walks the tensors its range overlaps; each
// thread owns one octet per iteration (128-bit loads/stores when aligned).

#include "luma_b200.h"
#include "luma_internal.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <type_traits>

static_assert(sizeof(LumaTensorDesc) == 96, "LumaTensorDesc layout");
static_assert(sizeof(LumaStepRow) == 56, "LumaStepRow layout");
static_assert(sizeof(LumaGrid) == 64, "LumaGrid layout");
static_assert(sizeof(LumaSlot) == 144, "LumaSlot layout");
static_assert(sizeof(LumaStepArgs) == 104, "LumaStepArgs layout");

namespace {

constexpr int kThreads = 256;           // luma_decode
constexpr int kThreadsPass1 = 1024;     // one CTA per SM (128 KB decode table)
constexpr int kThreadsPass2 = 512;      // one CTA per SM, <= 128 registers, 2 pairs per
                                        // thread per iteration (measured best)
constexpr int kMaxWarps = 32;

// Decode table of expm1f(fl(|q| * delta_m)) for |q| = 0..32768, built in
// shared memory when a CTA's segment of a tensor is long enough to repay the
// 32769 expm1f evaluations.  Same function on the same inputs, so lookups are
// bit-identical to evaluating expm1f.
constexpr int kLutEntries = 32769;
constexpr int64_t kLutMinElems = 131072;
constexpr size_t kLutBytes = kLutEntries * sizeof(float);

// Pass-2 steady loop: each thread steps two pairs per iteration and stages
// the raw words of its next pairs in shared memory with asynchronous copies,
// kHotStages pair slots deep (kHotStages / 2 - 1 iterations ahead), after the
// decode table.  A slot holds, per thread, up to 8 bytes of param, 8 of grad,
// 4 of Q_m and 4 of Q_w.
#ifndef LUMA_HOT_STAGES
#define LUMA_HOT_STAGES 4
#endif
constexpr int kHotStages = LUMA_HOT_STAGES;
constexpr size_t kLutPadBytes = (kLutBytes + 127) / 128 * 128;
constexpr size_t kHotStageBytes = (size_t)kThreadsPass2 * 24;
constexpr size_t kPass2SmemBytes = kLutPadBytes + kHotStages * kHotStageBytes;
// Pass-1 staging (quantized steps of aligned tensors): per thread one quad
// (4 elements) per stage: up to 16 bytes of grad, 8 of Q_m, 8 of Q_w.
#ifndef LUMA_P1_STAGES
#define LUMA_P1_STAGES 2
#endif
constexpr int kP1Stages = LUMA_P1_STAGES;
// Staged pass-1 loop: iterations between exchanges of the warp's bounds.
#ifndef LUMA_P1_SYNC_EVERY
#define LUMA_P1_SYNC_EVERY 8
#endif
constexpr int kP1SyncEvery = LUMA_P1_SYNC_EVERY;
constexpr size_t kP1StageBytes = (size_t)kThreadsPass1 * 32;
constexpr size_t kPass1SmemBytes = kLutPadBytes + kP1Stages * kP1StageBytes;

// Pass-1 accumulators of one tensor (the amax_m / amax_v / done fields of a
// LumaSlot) for luma_step_noalloc, which keeps them in the library's own
// static device array instead of the caller's slots.
struct PassAccum {
  uint32_t amax_m;
  uint32_t amax_v;
  unsigned long long done;
};
static_assert(sizeof(PassAccum) == 16, "PassAccum layout");

// Scratch of luma_step_noalloc: LUMA_NOALLOC_MAX_DESCS x 16 bytes, part of the
// module image, so every GPU that loads the library holds it until exit.
// Host code must not use this name as a device address; the set-up in
// noalloc_scratch() fetches the address with cudaGetSymbolAddress.
static __device__ __align__(256) PassAccum g_noalloc_accum[LUMA_NOALLOC_MAX_DESCS];

// LUMA_KERR_* flags raised by the kernels (read by luma_error_flags).
static __device__ unsigned int g_kernel_error = 0u;

// ---------------------------------------------------------------------------
// Error reporting
// ---------------------------------------------------------------------------

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(luma_g_err, sizeof(luma_g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(LUMA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// ---------------------------------------------------------------------------
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel Random Numbers: As Easy
// as 1, 2, 3", SC'11): 10 rounds of two 32x32->64 multiplies with the key
// bumped by the Weyl constants between rounds.
// ---------------------------------------------------------------------------

constexpr uint32_t kPhiloxM0 = 0xD2511F53u;
constexpr uint32_t kPhiloxM1 = 0xCD9E8D57u;
constexpr uint32_t kPhiloxW0 = 0x9E3779B9u;
constexpr uint32_t kPhiloxW1 = 0xBB67AE85u;

// The 32x32 -> 64-bit products are written as one 64-bit multiply each (one
// wide multiply instruction instead of separate low and high halves).
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)kPhiloxM0 * c.x;
    const uint64_t p1 = (uint64_t)kPhiloxM1 * c.z;
    c = make_uint4((uint32_t)(p1 >> 32) ^ c.y ^ k0, (uint32_t)p1, (uint32_t)(p0 >> 32) ^ c.w ^ k1,
                   (uint32_t)p0);
    k0 += kPhiloxW0;
    k1 += kPhiloxW1;
  }
  return c;
}

// Two Philox4x32-10 blocks with the same key, interleaved: the key schedule
// is computed once for both and the two dependency chains overlap.
__device__ __forceinline__ void philox_x2(uint4& a, uint4& b, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint64_t pa0 = (uint64_t)kPhiloxM0 * a.x, pa1 = (uint64_t)kPhiloxM1 * a.z;
    const uint64_t pb0 = (uint64_t)kPhiloxM0 * b.x, pb1 = (uint64_t)kPhiloxM1 * b.z;
    a = make_uint4((uint32_t)(pa1 >> 32) ^ a.y ^ k0, (uint32_t)pa1,
                   (uint32_t)(pa0 >> 32) ^ a.w ^ k1, (uint32_t)pa0);
    b = make_uint4((uint32_t)(pb1 >> 32) ^ b.y ^ k0, (uint32_t)pb1,
                   (uint32_t)(pb0 >> 32) ^ b.w ^ k1, (uint32_t)pb0);
    k0 += kPhiloxW0;
    k1 += kPhiloxW1;
  }
}

// Top 24 bits of a Philox word: the uniform u = (x >> 8) * 2^-24 in [0, 1),
// kept scaled by 2^24 (an exact integer-valued float).  The LogSR decision
// u < p* is evaluated as U < p* * 2^24; scaling by a power of two is exact.
__device__ __forceinline__ float u24_scaled(uint32_t x) {
  return __uint2float_rn(x >> 8);
}

// ---------------------------------------------------------------------------
// Grid precompute, float64 on device (reference functional.py:74-92).
// ---------------------------------------------------------------------------

__device__ void make_grid(double S_m, double S_v, double eps, LumaGrid* g) {
  const double w_min = 1.0 / (sqrt(S_v) + eps);
  const double delta_m = log1p(S_m) / (double)LUMA_K_M;
  const double z_m = expm1(delta_m);
  const double ratio = 1.0 / (eps * w_min);
  const double delta_w = (ratio > 1.0) ? log(ratio) / (double)LUMA_K_W : 0.0;
  const double z_w = (delta_w > 0.0) ? expm1(delta_w) : 1.0;
  g->S_m = S_m;
  g->S_v = S_v;
  g->eps = eps;
  // A float32 tensor divided by a Python scalar s is multiplied by
  // fl32(1.0 / s) on CUDA, the reciprocal taken in float64.
  g->dm = __double2float_rn(delta_m);
  g->inv_dm = __double2float_rn(1.0 / delta_m);
  g->inv_zm = __double2float_rn(1.0 / z_m);
  g->s_m32 = __double2float_rn(S_m);
  g->w_min = __double2float_rn(w_min);
  g->inv_wmin = __double2float_rn(1.0 / w_min);
  g->dw = __double2float_rn(delta_w);
  g->inv_dw = (delta_w > 0.0) ? __double2float_rn(1.0 / delta_w) : 0.0f;
  g->inv_zw = __double2float_rn(1.0 / z_w);
  g->dw_pos = (delta_w > 0.0) ? 1 : 0;
}

// ---------------------------------------------------------------------------
// Element arithmetic.  Every helper names the reference expression it
// evaluates; each torch op of the reference is one correctly rounded fp32 op.
// ---------------------------------------------------------------------------

// Clamps below keep NaN inputs as ATen's clamp kernels do (a NaN operand
// fails every comparison and passes through the select unchanged).

// Per-thread asynchronous global -> shared copies (cp.async, 4 or 8 bytes;
// completion tracked per thread with commit / wait groups).
template <int kBytes>
__device__ __forceinline__ void cp_async(void* smem_dst, const void* gmem_src) {
  static_assert(kBytes == 4 || kBytes == 8 || kBytes == 16, "cp.async size");
  if constexpr (kBytes == 16) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::
                     "r"((uint32_t)__cvta_generic_to_shared(smem_dst)), "l"(gmem_src)
                 : "memory");
  } else {
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::
                     "r"((uint32_t)__cvta_generic_to_shared(smem_dst)), "l"(gmem_src), "n"(kBytes)
                 : "memory");
  }
}

__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int kPending>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(kPending) : "memory");
}

struct Consts {
  // step row
  float beta1, omb1, beta2, omb2, decay, neg_eta, inv_bc2, eps32, w_max;
  // fused grad scaling (clip_grad_norm_'s coefficient), has_gscale != 0
  float gscale;
  int has_gscale;
  // pass 1 flags non-finite grads (LumaStepArgs.found_inf != NULL)
  int check_inf;
  // decode grid (codes as stored)
  float o_dm, o_wmin, o_dw;
  // encode grid (this step's new scales), pass 2 only
  float n_sm32, n_dm, n_inv_dm, n_inv_zm, n_wmin, n_inv_wmin, n_dw, n_inv_dw, n_inv_zw;
  int n_dw_pos;
  int init;
  // LogSR decision on uniforms scaled by 2^24: inv_z * 2^24, and margins
  // kDecisionMargin * 2^24 where the series is valid, 2^25 (always the exact
  // path) where delta is too large for it
  float inv_zm24, inv_zw24, margin_m, margin_w;
  // pass-1 approximate decode
  float o_dw_log2e;
  float tau_v;  // kBoundEps * eps^2
};

// m = sgn(Q_m) * expm1(|Q_m| * delta_m)       functional.py:113-116
__device__ __forceinline__ float decode_m(int q, float dm) {
  const float e = expm1f(__fmul_rn((float)abs(q), dm));
  return q < 0 ? -e : e;
}

__device__ __forceinline__ float decode_m_lut(int q, const float* lut) {
  const float e = lut[abs(q)];
  return q < 0 ? -e : e;
}

// w = w_min * exp(Q_w * delta_w)               functional.py:119-126
// v = (1.0 / w - eps).clamp_min(0).square()    functional.py:270
__device__ __forceinline__ float decode_v(uint32_t qu, float wmin, float dw, float eps32) {
  const float w = __fmul_rn(wmin, expf(__fmul_rn((float)qu, dw)));
  float t = __fsub_rn(__frcp_rn(w), eps32);
  t = t < 0.0f ? 0.0f : t;  // clamp_min(0), NaN kept
  return __fmul_rn(t, t);
}

// m' = beta1 * m + (1 - beta1) * g ;  v' = beta2 * v + (1 - beta2) * g^2
// (functional.py:274-275; first step functional.py:204-205 with m = v = 0).
__device__ __forceinline__ void ema(const Consts& c, float g, float m, float v,
                                    float& mn, float& vn) {
  const float g2 = __fmul_rn(g, g);
  if (c.init) {
    mn = __fmul_rn(c.omb1, g);
    vn = __fmul_rn(c.omb2, g2);
  } else {
    mn = __fadd_rn(__fmul_rn(c.beta1, m), __fmul_rn(c.omb1, g));
    vn = __fadd_rn(__fmul_rn(c.beta2, v), __fmul_rn(c.omb2, g2));
  }
}

// Whether any of the n loaded grad values is inf or NaN (exponent all ones):
// the test torch._amp_foreach_non_finite_check_and_unscale_ applies to each
// grad element before unscaling it.
template <int N>
__device__ __forceinline__ int any_nonfinite(const float (&g)[N]) {
  int bad = 0;
#pragma unroll
  for (int j = 0; j < N; ++j) bad |= (__float_as_uint(g[j]) & 0x7F800000u) == 0x7F800000u;
  return bad;
}

// Fused grad scaling: g -> round_to_grad_dtype(fl32(g) * c), what
// torch._foreach_mul_(grads, c) stores (clip_grad_norm_'s last step).
template <int GD>
__device__ __forceinline__ float scale_grad(float g, float c) {
  const float x = __fmul_rn(g, c);
  if (GD == LUMA_F32) return x;
  if (GD == LUMA_BF16) return __bfloat162float(__float2bfloat16_rn(x));
  return __half2float(__float2half_rn(x));
}

template <int GD, int N>
__device__ __forceinline__ void scale_grads(const Consts& c, float (&g)[N]) {
  if (c.has_gscale) {
#pragma unroll
    for (int j = 0; j < N; ++j) g[j] = scale_grad<GD>(g[j], c.gscale);
  }
}

template <int GD>
__device__ __forceinline__ void scale_grads2(const Consts& c, float& g0, float& g1) {
  if (c.has_gscale) {
    g0 = scale_grad<GD>(g0, c.gscale);
    g1 = scale_grad<GD>(g1, c.gscale);
  }
}

// param.mul_(1 - wd*lr); param.addcdiv_(m', sqrt(v'/bc2) + eps, value=-eta)
// (functional.py:278-279, 213-214).  v'/bc2 is v' * fl32(1.0/bc2) on
// CUDA; addcdiv is fma(value, m'/den, param).
__device__ __forceinline__ float adamw(const Consts& c, float p, float mn, float vn) {
  const float pd = __fmul_rn(p, c.decay);
  const float den = __fadd_rn(__fsqrt_rn(__fmul_rn(vn, c.inv_bc2)), c.eps32);
  return __fmaf_rn(c.neg_eta, __fdiv_rn(mn, den), pd);
}

// ---------------------------------------------------------------------------
// Branch-free correctly rounded reciprocal, square root and quotient for the
// steady-state loop.  CUDA's IEEE __frcp_rn / __fsqrt_rn / __fdiv_rn each test
// their operands and branch to a slow path; those branches split the loop body
// into small blocks.  The forms below start from the hardware approximations
// and apply the FMA residual corrections of Markstein's method (P. Markstein,
// "Computation of elementary functions on the IBM RISC System/6000 processor",
// IBM J. Res. Dev. 34(1), 1990).  Each is correctly rounded (round to nearest
// even, the result of the IEEE intrinsic) on the operand range stated, which
// was established by exhaustive comparison with the intrinsic on a B200:
//   rcp_cr(b):    every float with 2^-125 <= |b| <= 2^125;
//   sqrt_cr(x):   every float with 2^-102 <= x <= FLT_MAX;
//   div_cr(a, b): every pair of significands (a, b in [1, 2): 2^46 pairs) and
//                 2^36 random pairs with 2^-100 <= |a|, |b| < 2^100 and the
//                 quotient in [2^-120, 2^120] (exponents only scale the
//                 intermediate values while they stay normal).
// Outside those ranges the caller must use the IEEE intrinsics;
// luma_arith_selfcheck() repeats the comparison on the current GPU.
// ---------------------------------------------------------------------------

__device__ __forceinline__ float rcp_approx_ftz(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float rsqrt_approx_ftz(float x) {
  float y;
  asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 1/b: one Newton-Raphson step y0 + y0 (1 - b y0), the residual exact in an FMA.
__device__ __forceinline__ float rcp_cr(float b) {
  const float y0 = rcp_approx_ftz(b);
  return __fmaf_rn(y0, __fmaf_rn(-b, y0, 1.0f), y0);
}

// sqrt(x): s0 = x rsqrt(x), corrected once by the exact residual x - s0^2
// times 1/(2 sqrt(x)).
__device__ __forceinline__ float sqrt_cr(float x) {
  const float r0 = rsqrt_approx_ftz(x);
  const float s0 = __fmul_rn(x, r0);
  return __fmaf_rn(__fmaf_rn(-s0, s0, x), __fmul_rn(0.5f, r0), s0);
}

// a/b: q0 = a RN(1/b), corrected once by the exact residual a - b q0.
__device__ __forceinline__ float div_cr(float a, float b) {
  const float y = rcp_cr(b);
  const float q0 = __fmul_rn(a, y);
  return __fmaf_rn(__fmaf_rn(-b, q0, a), y, q0);
}

// ---------------------------------------------------------------------------
// Certified logarithms of the steady pass-2 loop.  The codes depend on
// y = fl(log1pf(a) * inv_dm) (momentum) and y = fl(logf(z) * inv_dw)
// (preconditioner) only through floor(y) and the LogSR decision, and both are
// monotone in y.  So y is first taken from a cheap approximation L~ of the
// logarithm whose distance to CUDA's own result is bounded:
//   |log1pf(a) - log1p_series(a)| <= kLog1pRel * log1p_series(a)   a in [0, 2^-5]
//   |logf(z) - log_approx(z)| <= kLogAbs + kLogRel * |log_approx(z)|
//                                                             z in [2^-1, 2^64]
// (verified exhaustively, every float of both domains, by luma_log_selfcheck).
// Then every y CUDA's functions can produce lies within dy of fl(L~ * inv);
// if that interval decides floor(y) and the decision, the code is the exact
// one; otherwise the element is finished by the exact functions.
// ---------------------------------------------------------------------------

constexpr float kCertLog1pMax = 0x1.0p-5f;
constexpr float kCertLogZMin = 0x1.0p-1f;
constexpr float kCertLogZMax = 0x1.0p64f;
constexpr float kLog1pRel = 0x1.0p-21f;
constexpr float kLogAbs = 0x1.0p-22f;
constexpr float kLogRel = 0x1.0p-22f;

// log1p(a) = a - a^2/2 + a^3/3 - a^4/4 + a^5/5 - a^6/6 + ...: for a <= 2^-5
// the omitted terms are below a * 2^-30 / 7.
__device__ __forceinline__ float log1p_series(float a) {
  float p = __fmaf_rn(a, -1.0f / 6.0f, 0.2f);
  p = __fmaf_rn(a, p, -0.25f);
  p = __fmaf_rn(a, p, 1.0f / 3.0f);
  p = __fmaf_rn(a, p, -0.5f);
  p = __fmaf_rn(a, p, 1.0f);
  return __fmul_rn(a, p);
}

// ln z = log2(z) * ln 2 with the hardware log2 approximation (MUFU).
__device__ __forceinline__ float log_approx(float z) {
  float l2;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(l2) : "f"(z));
  return __fmul_rn(l2, 0.693147182f);
}

// LogSR decision  u < p*,  p* = fl(expm1f(fl(frac * delta)) * inv_z)
// (functional.py:64-66).  For delta <= kSeriesMaxDelta the series
// x + x^2/2 + x^3/6 (x = fl(frac * delta) <= delta) is within 3e-7 of p*:
// expm1f is within 1 ulp, the omitted x^4/24 term is below 6e-8 relative,
// and the roundings add under 2 ulp.  Only when u falls within the margin
// (kDecisionMargin, 6x that bound) of the series value is expm1f evaluated,
// so the decision, and therefore the code, is the one the exact expression
// gives.  Any finite float64 grid has delta_m <= 0.0028 and delta_w <= 0.0109;
// beyond kSeriesMaxDelta the margin is 2, which sends every element to the
// exact expression.
constexpr float kSeriesMaxDelta = 0.011f;
constexpr float kDecisionMargin = 0x1.0p-19f;
constexpr float kUScale = 0x1.0p24f;

// Margin on the 2^24-scaled scale.
__host__ __device__ __forceinline__ float decision_margin(float delta) {
  return delta <= kSeriesMaxDelta ? kDecisionMargin * kUScale : 2.0f * kUScale;
}

// U = u * 2^24; inv_z24 = inv_z * 2^24; margin24 from decision_margin().
// The series value and U are below 2^24, so the subtraction adds at most
// 0.5 to the 5 (= 3e-7 * 2^24) series error bound, against a margin of 32.
__device__ __forceinline__ bool logsr_up(float fr, float delta, float inv_z, float inv_z24,
                                         float U, float margin24) {
  const float x = __fmul_rn(fr, delta);
  const float e = __fmaf_rn(__fmul_rn(x, x), __fmaf_rn(x, 1.0f / 6.0f, 0.5f), x);
  const float diff = __fsub_rn(U, __fmul_rn(e, inv_z24));
  if (fabsf(diff) > margin24) return diff < 0.0f;
  return U < __fmul_rn(__fmul_rn(expm1f(x), inv_z), kUScale);
}

// The steady pass-2 loop evaluates the same series as one polynomial in the
// fraction fr = y - floor(y) with the scalings folded into its coefficients:
//   E = fr (c1 + fr (c2 + fr c3)),  c1 = d K, c2 = d^2 K / 2, c3 = d^3 K / 6,
//   K = inv_z * 2^24 (d = fl32(delta), the factor of x = fl(fr * d)),
// and takes diff = fl(U - E) in one FMA.  Against P = p* * 2^24 of the
// reference expression: |P - S(x) K| <= 5 as above (the rounding of x moves
// p* by at most 2^-24 relative, one more unit); the coefficients, rounded
// from float64, and the three roundings of the evaluation add at most 6
// relative ulps of E <= 2^24, i.e. 6; the final rounding at most 1.  So
// |diff - (U - P)| <= 13 < 32 (the margin): whenever |diff| > 32 its sign is
// the sign of U - P, the exact decision.
// Where delta > kSeriesMaxDelta the coefficients are NaN instead, so that
// every decision of the segment is undecided (|NaN| > margin is false) and the
// margin of the steady loop is the constant kHotMargin.
constexpr float kHotMargin = kDecisionMargin * kUScale;  // 32

__device__ __forceinline__ void series_coefs(float d, float inv_z, float& c1, float& c2,
                                             float& c3) {
  const double k = (double)inv_z * (double)kUScale, x = (double)d;
  const bool ok = d <= kSeriesMaxDelta;  // false for NaN
  c1 = ok ? (float)(x * k) : __int_as_float(0x7FC00000);
  c2 = (float)(x * x * k * 0.5);
  c3 = (float)(x * x * x * k / 6.0);
}

// _quantize_momentum (functional.py:133-150) with _log_sr (functional.py:38-67).
// |m.clamp(-S_m, S_m)| = min(|m|, S_m) (NaN kept); y >= 0 because log1pf of a
// non-negative value is non-negative, so of clamp(0, K_M) only the upper bound
// can bite; sign(m_clip) * q is applied to the integer (for m = 0, q = 0).
__device__ __forceinline__ int quant_m(const Consts& c, float mn, float U) {
  const float a = fabsf(mn);
  const float ac = a > c.n_sm32 ? c.n_sm32 : a;
  const float y = __fmul_rn(log1pf(ac), c.n_inv_dm);
  const float fy = floorf(y);
  const float fr = __fsub_rn(y, fy);
  float r = __fadd_rn(fy, logsr_up(fr, c.n_dm, c.n_inv_zm, c.inv_zm24, U, c.margin_m) ? 1.0f : 0.0f);
  r = r > (float)LUMA_K_M ? (float)LUMA_K_M : r;
  const int ri = (int)r;
  return mn < 0.0f ? -ri : ri;
}

// _quantize_preconditioner (functional.py:153-176) with _log_sr.  v' >= 0 (or
// NaN), so v'.clamp_min(0) is the identity.
__device__ __forceinline__ uint32_t quant_w(const Consts& c, float vn, float U) {
  // delta_w == 0 (_log_sr returns 0): inv_dw = 0 makes y = 0, frac = 0 and
  // p* = 0, so the expression below yields 0 without a branch.
  const float den = __fadd_rn(__fsqrt_rn(vn), c.eps32);
  float w = __frcp_rn(den);
  w = w < c.n_wmin ? c.n_wmin : (w > c.w_max ? c.w_max : w);  // clamp, NaN kept
  const float y = __fmul_rn(logf(__fmul_rn(w, c.n_inv_wmin)), c.n_inv_dw);
  const float fy = floorf(y);
  const float fr = __fsub_rn(y, fy);
  float r = __fadd_rn(fy, logsr_up(fr, c.n_dw, c.n_inv_zw, c.inv_zw24, U, c.margin_w) ? 1.0f : 0.0f);
  r = r < 0.0f ? 0.0f : (r > (float)LUMA_K_W ? (float)LUMA_K_W : r);  // clamp(0, K_W), NaN kept
  return (uint32_t)(int)r;  // .to(int32) then two's-complement wrap to int16
}

// ---------------------------------------------------------------------------
// Pass-1 maxima with certified bounds.
//
// The new scales need the exact max |m'| and max v' of a tensor, but only the
// maximal elements need their exact values.  Pass 1 evaluates every element
// with a cheap approximate decode whose error is bounded (below), keeps a
// running lower bound T of the maximum (warp-wide), and evaluates exactly only
// elements whose upper bound exceeds both T and the exact maximum found so
// far.  An element that is skipped has a value strictly below some other
// element's exact value, so the exact maximum is unchanged.  NaN and
// infinite approximations always take the exact path.
//
// Approximate decode, relative errors:
//   expm1(x): x + x^2 (1/2 + x (1/6 + x/24)) for x < 0.125 (truncation < 2.1e-6),
//             ex2.approx(x log2 e) - 1 otherwise (< 1e-5 up to x = 88.7, the
//             largest |q| delta_m a float32 scale allows);
//   v:        ex2.approx of an argument up to 128 (log2 of the grid ratio) with
//             three roundings (< 1.6e-5), rcp.approx, then t = 1/w - eps:
//             |v~ - v| < 2e-5 (v + t eps), t eps <= (v + eps^2) / 2.
// Bounds, with kBoundEps = 2^-13 (>= 4x the errors above):
//   | |m'~| - |m'| | <= kBoundEps (|beta1 m~| + |m'~|) + 2^-147   (q != 0)
//   |  v'~ - v'    | <= kBoundEps  v'~ + kBoundEps eps^2 + 2^-147
// The 2^-147 term covers roundings of subnormal intermediates.  For q == 0
// (or beta1 == 0) m' = fl(c1 g) exactly and is taken as is.
// ---------------------------------------------------------------------------

constexpr float kBoundEps = 0x1.0p-13f;
constexpr float kTinyAbs = 0x1.0p-147f;

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float expm1_approx(float x) {
  const float series = __fmaf_rn(__fmul_rn(x, x),
                                 __fmaf_rn(x, __fmaf_rn(x, 1.0f / 24.0f, 1.0f / 6.0f), 0.5f), x);
  return x < 0.125f ? series : ex2_approx(x * 1.44269504f) - 1.0f;
}

// ---------------------------------------------------------------------------
// Octet loads and stores
// ---------------------------------------------------------------------------

template <int DT>
__device__ __forceinline__ void load8(const void* base, int64_t e0, int n, bool vec, float (&x)[8]) {
  if (DT == LUMA_F32) {
    const float* p = static_cast<const float*>(base) + e0;
    if (vec) {
      const float4 a = __ldcs(reinterpret_cast<const float4*>(p));
      const float4 b = __ldcs(reinterpret_cast<const float4*>(p) + 1);
      x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
      x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) x[j] = (j < n) ? p[j] : 0.0f;
    }
  } else {
    const uint16_t* p = static_cast<const uint16_t*>(base) + e0;
    uint16_t h[8];
    if (vec) {
      const uint4 a = __ldcs(reinterpret_cast<const uint4*>(p));
      memcpy(h, &a, 16);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) h[j] = (j < n) ? p[j] : (uint16_t)0;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (DT == LUMA_BF16) {
        x[j] = __uint_as_float((uint32_t)h[j] << 16);  // bf16 -> f32 is exact
      } else {
        x[j] = __half2float(__ushort_as_half(h[j]));
      }
    }
  }
}

__device__ __forceinline__ void load8_codes(const int16_t* base, int64_t e0, int n, bool vec,
                                            uint16_t (&q)[8]) {
  const uint16_t* p = reinterpret_cast<const uint16_t*>(base) + e0;
  if (vec) {
    const uint4 a = __ldcs(reinterpret_cast<const uint4*>(p));
    memcpy(q, &a, 16);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) q[j] = (j < n) ? p[j] : (uint16_t)0;
  }
}

template <int DT>
__device__ __forceinline__ void store8(void* base, int64_t e0, int n, bool vec, const float (&x)[8]) {
  if (DT == LUMA_F32) {
    float* p = static_cast<float*>(base) + e0;
    if (vec) {
      __stcs(reinterpret_cast<float4*>(p), make_float4(x[0], x[1], x[2], x[3]));
      __stcs(reinterpret_cast<float4*>(p) + 1, make_float4(x[4], x[5], x[6], x[7]));
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j < n) p[j] = x[j];
    }
  } else {  // bf16, round to nearest even
    uint16_t* p = static_cast<uint16_t*>(base) + e0;
    uint16_t h[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) h[j] = __bfloat16_as_ushort(__float2bfloat16_rn(x[j]));
    if (vec) {
      uint4 a;
      memcpy(&a, h, 16);
      __stcs(reinterpret_cast<uint4*>(p), a);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j < n) p[j] = h[j];
    }
  }
}

// ---------------------------------------------------------------------------
// Per-tensor segment bodies
// ---------------------------------------------------------------------------

// Per-segment state in shared memory: descriptor, step row, decode grid (of
// the previous step) and encode grid (of this step).
struct SegShared {
  LumaTensorDesc d;
  LumaStepRow row;
  LumaGrid dec;
  LumaGrid enc;
  int64_t next_pos;
  int skip;  // capturable mode: the step's row is outside the table
  int has_gscale;  // grads are scaled by gscale (LumaStepArgs.grad_scale)
  float gscale;
  int check_inf;   // pass 1 looks for inf / NaN grads (LumaStepArgs.found_inf)
  // pass 2: the series of the steady loop's LogSR decisions folded into one
  // polynomial in frac per code (series_coefs of the encode grid)
  float pm1, pm2, pm3, pw1, pw2, pw3;
};

// The CTA's segment state and decode table.  At namespace scope so that the
// out-of-line segment functions address them as shared memory.
__shared__ SegShared g_seg;
extern __shared__ float g_lut[];  // kLutEntries floats when launched with the table

__device__ __forceinline__ void fill_consts(const SegShared& s, bool pass2, Consts& c) {
  c.beta1 = s.row.beta1; c.omb1 = s.row.omb1; c.beta2 = s.row.beta2; c.omb2 = s.row.omb2;
  c.decay = s.row.decay; c.neg_eta = s.row.neg_eta; c.inv_bc2 = s.row.inv_bc2;
  c.eps32 = s.row.eps32; c.w_max = s.row.w_max;
  c.init = (s.row.step == 1) ? 1 : 0;
  c.gscale = s.gscale;
  c.has_gscale = s.has_gscale;
  c.check_inf = s.check_inf;
  c.o_dm = s.dec.dm; c.o_wmin = s.dec.w_min; c.o_dw = s.dec.dw;
  if (pass2) {
    c.n_sm32 = s.enc.s_m32; c.n_dm = s.enc.dm; c.n_inv_dm = s.enc.inv_dm; c.n_inv_zm = s.enc.inv_zm;
    c.n_wmin = s.enc.w_min; c.n_inv_wmin = s.enc.inv_wmin; c.n_dw = s.enc.dw;
    c.n_inv_dw = s.enc.inv_dw; c.n_inv_zw = s.enc.inv_zw; c.n_dw_pos = s.enc.dw_pos;
    c.margin_m = decision_margin(c.n_dm);
    c.margin_w = decision_margin(c.n_dw);
    c.inv_zm24 = c.n_inv_zm * kUScale;
    c.inv_zw24 = c.n_inv_zw * kUScale;
  } else {
    c.o_dw_log2e = c.o_dw * 1.44269504f;
    c.tau_v = kBoundEps * c.eps32 * c.eps32 + kTinyAbs;
  }
}

// Running state of the pass-1 maximum search of one tensor segment.
//   am/av: this thread's exact max |m'| / max v' (float bit patterns);
//   Tm/Tv: warp-wide lower bounds of the maxima from earlier iterations;
//   lm/lv: this thread's running lower bounds (they include the element under
//          test, whose own bound never excludes it).
struct MaxSearch {
  uint32_t am = 0u, av = 0u;
  int bad = 0;  // a grad element seen by this thread is inf or NaN (check_inf)
  float Tm = 0.0f, Tv = 0.0f, lm = 0.0f, lv = 0.0f;

  // Fold the thread bounds, and the exact maxima (values of actual elements,
  // so lower bounds of the tensor's maxima), into the warp-wide ones (all 32
  // lanes call this).  fmaxf drops a NaN maximum; the clamp at 0 keeps the
  // reduced bit patterns those of non-negative floats.
  __device__ __forceinline__ void warp_sync_bounds() {
    const float xm = fmaxf(fmaxf(lm, __uint_as_float(am)), 0.0f);
    const float xv = fmaxf(fmaxf(lv, __uint_as_float(av)), 0.0f);
    Tm = fmaxf(Tm, __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(xm))));
    Tv = fmaxf(Tv, __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(xv))));
  }
};

// Packed 16-bit minima / maxima (two lanes per 32-bit word).
__device__ __forceinline__ uint32_t vmax_s16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.s16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t vmin_s16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("min.s16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t vmax_u16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t vmin_u16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("min.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// G = max |g| over the four staged grads of a quad, from their bit patterns:
// the largest magnitude pattern, so an inf or NaN grad makes G inf or NaN
// (NaN patterns order above inf).  `bad`: one of them is inf or NaN.
template <int GD>
__device__ __forceinline__ float quad_gmax(const unsigned char* s, int& bad) {
  if constexpr (GD == LUMA_F32) {
    const uint4 v = *reinterpret_cast<const uint4*>(s);
    const uint32_t b = max(max(v.x & 0x7FFFFFFFu, v.y & 0x7FFFFFFFu),
                           max(v.z & 0x7FFFFFFFu, v.w & 0x7FFFFFFFu));
    bad = b >= 0x7F800000u;
    return __uint_as_float(b);
  } else {
    const uint2 v = *reinterpret_cast<const uint2*>(s);
    const uint32_t h = vmax_u16x2(v.x & 0x7FFF7FFFu, v.y & 0x7FFF7FFFu);
    const uint32_t b = max(h & 0xFFFFu, h >> 16);
    if constexpr (GD == LUMA_BF16) {
      bad = b >= 0x7F80u;
      return __uint_as_float(b << 16);
    } else {
      bad = b >= 0x7C00u;
      return __half2float(__ushort_as_half((unsigned short)b));
    }
  }
}

// Whether a quad may hold the tensor's largest |m'| or v' above the running
// thresholds (pass 1, both tables present, decode table non-decreasing,
// bucket table non-increasing).  With G = max |g| (after the grad scaling),
// M = lut[max |q_m|] >= |m| and V = vbt[min q_w >> 8] >= v for all four
// elements, every rounded operation below is monotone in its operands, so
//   |m'| = |fl(fl(b1 m) + fl(c1 g))| <= fl(fl(b1 M) + fl(c1 G)) = ubm,
//   v'   =  fl(fl(b2 v) + fl(c2 fl(g g))) <= fl(fl(b2 V) + fl(c2 fl(G G))) = ubv.
// A quad with ubm <= thr_m and ubv <= thr_v (finite thresholds, each the value
// of an element already seen) cannot raise either maximum and is skipped.  A
// non-finite bound (inf / NaN grad or table entry) never compares <= a finite
// threshold, so such quads are always evaluated exactly.
__device__ __forceinline__ bool quad_may_raise(const Consts& c, const float* lut, const float* vbt,
                                               float G, uint2 qm, uint2 qw, float thr_m,
                                               float thr_v) {
  const uint32_t hi = vmax_s16x2(qm.x, qm.y), lo = vmin_s16x2(qm.x, qm.y);
  const int mx = max((int)(int16_t)(uint16_t)hi, (int)hi >> 16);
  const int mn = min((int)(int16_t)(uint16_t)lo, (int)lo >> 16);
  const float M = lut[max(mx, -mn)];
  const uint32_t w = vmin_u16x2(qw.x, qw.y);
  const float V = vbt[min(w & 0xFFFFu, w >> 16) >> 8];
  const float ubm = __fadd_rn(__fmul_rn(c.beta1, M), __fmul_rn(c.omb1, G));
  const float ubv = __fadd_rn(__fmul_rn(c.beta2, V), __fmul_rn(c.omb2, __fmul_rn(G, G)));
  return !(ubm <= thr_m) || !(ubv <= thr_v);
}

// One element of pass 1 (step >= 2): exact |m'| from the decode table when
// there is one, certified-bound candidates otherwise.  v': with the bucket
// table `vbt` (vbt[k] >= v(q) for every code q of bucket k = q >> 8), the
// upper bound ub = fl(fl(beta2 vbt[k]) + fl((1-beta2) g^2)) >= v' (each
// rounded op is monotone), so an element whose ub does not beat the exact
// maximum found so far (this thread's, or the warp's from earlier
// iterations) cannot raise it; otherwise v' is evaluated exactly.  Without
// the table, certified approximate bounds.
__device__ __forceinline__ void pass1_elem(const Consts& c, const float* lut, const float* vbt,
                                           float g, int q, uint32_t qw, MaxSearch& ms) {
  if (lut != nullptr) {
    // exact |m'| from the decode table (functional.py:274, 282)
    const float mne = __fadd_rn(__fmul_rn(c.beta1, decode_m_lut(q, lut)), __fmul_rn(c.omb1, g));
    ms.am = max(ms.am, __float_as_uint(fabsf(mne)));
  } else if (q == 0 || c.beta1 == 0.0f) {
    // fl(beta1 * 0) = 0, so m' = fl(c1 g) exactly
    const float mne = fabsf(__fmul_rn(c.omb1, g));
    ms.am = max(ms.am, __float_as_uint(mne));
    ms.lm = fmaxf(ms.lm, mne);
  } else {
    const float e = expm1_approx(__fmul_rn((float)abs(q), c.o_dm));
    const float bm = c.beta1 * (q < 0 ? -e : e);
    const float mn = fabsf(bm + c.omb1 * g);
    const float bnd_m = kBoundEps * (fabsf(bm) + mn) + kTinyAbs;
    const float um = mn + bnd_m;
    ms.lm = fmaxf(ms.lm, mn - bnd_m);
    if (!(um <= __uint_as_float(ms.am)) && !(um < fmaxf(ms.Tm, ms.lm))) {
      // exact |m'| (functional.py:274, 282)
      const float mx = decode_m(q, c.o_dm);
      const float mne = __fadd_rn(__fmul_rn(c.beta1, mx), __fmul_rn(c.omb1, g));
      ms.am = max(ms.am, __float_as_uint(fabsf(mne)));
    }
  }
  if (vbt != nullptr) {
    const float g2 = __fmul_rn(c.omb2, __fmul_rn(g, g));
    const float ub = __fadd_rn(__fmul_rn(c.beta2, vbt[qw >> 8]), g2);
    if (!(ub <= __uint_as_float(ms.av)) && !(ub <= ms.Tv)) {
      // exact v' (functional.py:270, 275, 282)
      const float vne = __fadd_rn(__fmul_rn(c.beta2, decode_v(qw, c.o_wmin, c.o_dw, c.eps32)), g2);
      ms.av = max(ms.av, __float_as_uint(vne));
      ms.lv = fmaxf(ms.lv, vne);  // exact, so a lower bound of the maximum
    }
    return;
  }
  const float w = c.o_wmin * ex2_approx((float)qw * c.o_dw_log2e);
  const float t = fmaxf(rcp_approx(w) - c.eps32, 0.0f);
  const float vn = c.beta2 * (t * t) + c.omb2 * (g * g);
  const float bnd_v = kBoundEps * vn + c.tau_v;
  const float uv = vn + bnd_v;
  ms.lv = fmaxf(ms.lv, vn - bnd_v);
  if (!(uv <= __uint_as_float(ms.av)) && !(uv < fmaxf(ms.Tv, ms.lv))) {
    // exact v' (functional.py:270, 275, 282)
    const float v = decode_v(qw, c.o_wmin, c.o_dw, c.eps32);
    const float vne = __fadd_rn(__fmul_rn(c.beta2, v), __fmul_rn(c.omb2, __fmul_rn(g, g)));
    ms.av = max(ms.av, __float_as_uint(vne));
  }
}

// pass1_elem for the four elements of a quad when both tables are present:
// the four bounds are tested first and one branch per quad takes the exact
// decode of the elements that need it (a skip is justified against the
// maxima at the start of the quad, which only grow).
__device__ __forceinline__ void pass1_quad_tables(const Consts& c, const float* lut,
                                                  const float* vbt, const float (&g)[4],
                                                  const uint32_t (&qmw)[2], const uint32_t (&qww)[2],
                                                  MaxSearch& ms) {
  float g2[4];
  bool need[4];
  bool any = false;
  const float amax = __uint_as_float(ms.av);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int q = (int)(int16_t)(uint16_t)(qmw[e >> 1] >> (16 * (e & 1)));
    const float mne = __fadd_rn(__fmul_rn(c.beta1, decode_m_lut(q, lut)), __fmul_rn(c.omb1, g[e]));
    ms.am = max(ms.am, __float_as_uint(fabsf(mne)));
    const uint32_t qw = (qww[e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
    g2[e] = __fmul_rn(c.omb2, __fmul_rn(g[e], g[e]));
    const float ub = __fadd_rn(__fmul_rn(c.beta2, vbt[qw >> 8]), g2[e]);
    need[e] = !(ub <= amax) && !(ub <= ms.Tv);
    any |= need[e];
  }
  if (any) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (need[e]) {
        const uint32_t qw = (qww[e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
        const float vne = __fadd_rn(__fmul_rn(c.beta2, decode_v(qw, c.o_wmin, c.o_dw, c.eps32)), g2[e]);
        ms.av = max(ms.av, __float_as_uint(vne));
        ms.lv = fmaxf(ms.lv, vne);
      }
    }
  }
}

// Pass 1 over octets [o_lo, o_hi): one octet per thread per iteration, loaded
// straight into registers (16-byte loads when aligned).  Staging tiles through
// shared memory with bulk copies measured slower on B200 (the block barriers
// per tile cost more than the latency they hide at 32 warps per SM), and so did
// prefetching the next octet into registers (it spilled).  All threads run the
// same number of iterations (warp reductions).
template <int GD>
__device__ __forceinline__ void pass1_octets(const LumaTensorDesc& d, const Consts& c,
                                             const float* lut, const float* vbt, int64_t o_lo,
                                             int64_t o_hi, MaxSearch& ms) {
  constexpr int kThreads = kThreadsPass1;
  if (c.init) {  // first step: m' = (1-b1) g, v' = (1-b2) g^2, cheap and exact
    for (int64_t o = o_lo + threadIdx.x; o < o_hi; o += kThreads) {
      const int64_t e0 = o * 8;
      const int64_t rem = d.numel - e0;
      const int n = rem < 8 ? (int)rem : 8;
      float g[8];
      load8<GD>(d.grad, e0, n, d.vec_ok != 0 && n == 8, g);
      if (c.check_inf) ms.bad |= any_nonfinite(g);  // padding lanes load 0
      scale_grads<GD>(c, g);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (j < n) {
          float mn, vn;
          ema(c, g[j], 0.0f, 0.0f, mn, vn);
          ms.am = max(ms.am, __float_as_uint(fabsf(mn)));
          ms.av = max(ms.av, __float_as_uint(vn));
        }
      }
    }
    return;
  }
  for (int64_t ob = o_lo; ob < o_hi; ob += kThreads) {
    const int64_t o = ob + threadIdx.x;
    const int64_t e0 = o * 8;
    int n = 0;
    if (o < o_hi) {
      const int64_t rem = d.numel - e0;
      n = rem < 8 ? (int)rem : 8;
    }
    if (n > 0) {
      const bool vec = d.vec_ok != 0 && n == 8;
      float g[8];
      uint16_t qm[8], qw[8];
      load8<GD>(d.grad, e0, n, vec, g);
      if (c.check_inf) ms.bad |= any_nonfinite(g);
      scale_grads<GD>(c, g);
      load8_codes(d.q_m, e0, n, vec, qm);
      load8_codes(d.q_w, e0, n, vec, qw);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j < n) pass1_elem(c, lut, vbt, g[j], (int)(int16_t)qm[j], (uint32_t)qw[j], ms);
    }
    ms.warp_sync_bounds();
  }
}

// Pass 1 over quads [q_lo, q_hi) (4 elements each, all complete) of an aligned
// tensor at step >= 2: each thread copies the grad, Q_m and Q_w words of its
// quad kP1Stages - 1 iterations ahead into its own shared-memory slots with
// cp.async, so memory latency is hidden without holding the words in
// registers.  All threads run the same number of iterations (warp reductions).
template <int GD>
__device__ __forceinline__ void pass1_staged(const LumaTensorDesc& d, const Consts& c,
                                             const float* lut, const float* vbt, bool qb,
                                             int64_t q_lo, int64_t q_hi, MaxSearch& ms) {
  constexpr int kThreads = kThreadsPass1;
  constexpr int kGB = GD == LUMA_F32 ? 16 : 8;  // grad bytes per quad
  unsigned char* stage0 = reinterpret_cast<unsigned char*>(g_lut) + kLutPadBytes;
  unsigned char* sg = stage0 + (size_t)threadIdx.x * 16;
  unsigned char* sm = stage0 + (size_t)kThreads * 16 + (size_t)threadIdx.x * 8;
  unsigned char* sw = stage0 + (size_t)kThreads * 24 + (size_t)threadIdx.x * 8;
  const unsigned char* gq = static_cast<const unsigned char*>(d.grad) + q_lo * kGB;
  const unsigned char* mq = reinterpret_cast<const unsigned char*>(d.q_m) + q_lo * 8;
  const unsigned char* wq = reinterpret_cast<const unsigned char*>(d.q_w) + q_lo * 8;
  const int64_t n = q_hi - q_lo;
  auto issue = [&](int64_t j, int st) {  // quad j (relative) into stage st
    if (j < n) {
      const size_t o = (size_t)st * kP1StageBytes;
      cp_async<kGB>(sg + o, gq + j * kGB);
      cp_async<8>(sm + o, mq + j * 8);
      cp_async<8>(sw + o, wq + j * 8);
    }
    cp_async_commit();
  };
#pragma unroll
  for (int k = 0; k < kP1Stages - 1; ++k) issue(threadIdx.x + (int64_t)k * kThreads, k);
  int st = 0;
  // Finite thresholds: the largest exact maxima known to this lane.  They
  // are refreshed after an exact evaluation and after each exchange of the
  // warp's bounds (every kP1SyncEvery iterations); a stale threshold is still
  // the value of an element seen, so it only skips fewer quads.
  float thr_m = fminf(fmaxf(__uint_as_float(ms.am), ms.Tm), FLT_MAX);
  float thr_v = fminf(fmaxf(__uint_as_float(ms.av), ms.Tv), FLT_MAX);
  int it = 0;
  for (int64_t jb = 0; jb < n; jb += kThreads) {
    const int64_t j = jb + threadIdx.x;
    issue(j + (int64_t)(kP1Stages - 1) * kThreads, st == 0 ? kP1Stages - 1 : st - 1);
    cp_async_wait<kP1Stages - 1>();  // quad j has landed
    const size_t o = (size_t)st * kP1StageBytes;
    bool exact = j < n;
    if (qb && exact) {  // one bound per quad; see quad_may_raise
      int bad;
      float G = quad_gmax<GD>(sg + o, bad);
      if (c.check_inf) ms.bad |= bad;
      if (c.has_gscale) G = fabsf(scale_grad<GD>(G, c.gscale));
      exact = quad_may_raise(c, lut, vbt, G, *reinterpret_cast<const uint2*>(sm + o),
                             *reinterpret_cast<const uint2*>(sw + o), thr_m, thr_v);
    }
    if (exact) {
      float g[4];
      if constexpr (GD == LUMA_F32) {
        const float4 v = *reinterpret_cast<const float4*>(sg + o);
        g[0] = v.x; g[1] = v.y; g[2] = v.z; g[3] = v.w;
      } else {
        const uint2 v = *reinterpret_cast<const uint2*>(sg + o);
        const uint32_t h[4] = {v.x & 0xFFFFu, v.x >> 16, v.y & 0xFFFFu, v.y >> 16};
#pragma unroll
        for (int e = 0; e < 4; ++e)
          g[e] = (GD == LUMA_BF16) ? __uint_as_float(h[e] << 16)
                                   : __half2float(__ushort_as_half((unsigned short)h[e]));
      }
      if (c.check_inf && !qb) ms.bad |= any_nonfinite(g);
      scale_grads<GD>(c, g);
      const uint2 qm = *reinterpret_cast<const uint2*>(sm + o);
      const uint2 qw = *reinterpret_cast<const uint2*>(sw + o);
      const uint32_t qmw[2] = {qm.x, qm.y}, qww[2] = {qw.x, qw.y};
      if (vbt != nullptr) {
        pass1_quad_tables(c, lut, vbt, g, qmw, qww, ms);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t wm = qmw[e >> 1] >> (16 * (e & 1));
          const uint32_t ww = (qww[e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
          pass1_elem(c, lut, vbt, g[e], (int)(int16_t)(uint16_t)wm, ww, ms);
        }
      }
      thr_m = fminf(fmaxf(__uint_as_float(ms.am), ms.Tm), FLT_MAX);
      thr_v = fminf(fmaxf(__uint_as_float(ms.av), ms.Tv), FLT_MAX);
    }
    st = st == kP1Stages - 1 ? 0 : st + 1;
    if (++it == kP1SyncEvery) {  // the same iteration count on every lane
      it = 0;
      ms.warp_sync_bounds();
      thr_m = fminf(fmaxf(__uint_as_float(ms.am), ms.Tm), FLT_MAX);
      thr_v = fminf(fmaxf(__uint_as_float(ms.av), ms.Tv), FLT_MAX);
    }
  }
  ms.warp_sync_bounds();
  cp_async_wait<0>();  // no copy left in flight into the stages
}

// Two consecutive elements (one Philox block) of a stream as floats.
template <int DT>
__device__ __forceinline__ void load2(const void* base, int64_t e, bool both, bool vec,
                                      float& x0, float& x1) {
  if (DT == LUMA_F32) {
    const float* p = static_cast<const float*>(base) + e;
    if (vec) {
      const float2 a = __ldcs(reinterpret_cast<const float2*>(p));
      x0 = a.x; x1 = a.y;
    } else {
      x0 = p[0]; x1 = both ? p[1] : 0.0f;
    }
  } else {
    const uint16_t* p = static_cast<const uint16_t*>(base) + e;
    uint32_t h0, h1;
    if (vec) {
      const uint32_t a = __ldcs(reinterpret_cast<const unsigned int*>(p));
      h0 = a & 0xFFFFu; h1 = a >> 16;
    } else {
      h0 = p[0]; h1 = both ? p[1] : 0u;
    }
    if (DT == LUMA_BF16) {
      x0 = __uint_as_float(h0 << 16);  // bf16 -> f32 is exact
      x1 = __uint_as_float(h1 << 16);
    } else {
      x0 = __half2float(__ushort_as_half((unsigned short)h0));
      x1 = __half2float(__ushort_as_half((unsigned short)h1));
    }
  }
}

template <int DT>
__device__ __forceinline__ void store2(void* base, int64_t e, bool both, bool vec, float x0, float x1) {
  if (DT == LUMA_F32) {
    float* p = static_cast<float*>(base) + e;
    if (vec) {
      __stcs(reinterpret_cast<float2*>(p), make_float2(x0, x1));
    } else {
      p[0] = x0;
      if (both) p[1] = x1;
    }
  } else {  // bf16, round to nearest even
    uint16_t* p = static_cast<uint16_t*>(base) + e;
    const uint32_t h0 = __bfloat16_as_ushort(__float2bfloat16_rn(x0));
    const uint32_t h1 = __bfloat16_as_ushort(__float2bfloat16_rn(x1));
    if (vec) {
      __stcs(reinterpret_cast<unsigned int*>(p), h0 | (h1 << 16));
    } else {
      p[0] = (uint16_t)h0;
      if (both) p[1] = (uint16_t)h1;
    }
  }
}

__device__ __forceinline__ void store2_codes(int16_t* base, int64_t e, bool both, bool vec,
                                             uint32_t q0, uint32_t q1) {
  uint16_t* p = reinterpret_cast<uint16_t*>(base) + e;
  if (vec) {
    __stcs(reinterpret_cast<unsigned int*>(p), (q0 & 0xFFFFu) | (q1 << 16));
  } else {
    p[0] = (uint16_t)q0;
    if (both) p[1] = (uint16_t)q1;
  }
}

// Updated params through the multicast (NVLS) address of the param
// (LumaTensorDesc.param_mc): one multimem store per pair, replicated by the
// NVSwitch to every GPU bound to the multicast object.  Multimem stores are 32
// bits wide at least: a bf16 pair is one 32-bit word (for a lone last element
// the word's upper half, padding the caller owns, is written with zero); an
// fp32 pair is one 64-bit vector store.
__device__ __forceinline__ void mc_store_b32(void* addr, uint32_t v) {
  asm volatile("multimem.st.relaxed.sys.global.b32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ void mc_store_f32x2(void* addr, float a, float b) {
  asm volatile("multimem.st.relaxed.sys.global.v2.f32 [%0], {%1, %2};" ::"l"(addr), "f"(a), "f"(b)
               : "memory");
}

template <int PD>
__device__ __forceinline__ void mc_store2(void* base, int64_t e, bool both, float x0, float x1) {
  if (PD == LUMA_F32) {
    float* p = static_cast<float*>(base) + e;
    if (both) {
      mc_store_f32x2(p, x0, x1);
    } else {
      mc_store_b32(p, __float_as_uint(x0));
    }
  } else {
    uint16_t* p = static_cast<uint16_t*>(base) + e;
    const uint32_t h0 = __bfloat16_as_ushort(__float2bfloat16_rn(x0));
    const uint32_t h1 = both ? (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(x1)) : 0u;
    mc_store_b32(p, h0 | (h1 << 16));
  }
}

// The updated param pair: to the multicast address when the descriptor has
// one, and to the param itself unless the multicast address maps it.
template <int PD>
__device__ __forceinline__ void store_param2(const LumaTensorDesc& d, int64_t e, bool both,
                                             bool vec, float x0, float x1) {
  if (d.param_mc != nullptr) mc_store2<PD>(d.param_mc, e, both, x0, x1);
  if (d.param_mc == nullptr || d.mc_local) store2<PD>(d.param, e, both, vec, x0, x1);
}

// One element of pass 2: decode, EMA, AdamW, re-quantize.
__device__ __forceinline__ void pass2_elem(const Consts& c, const float* lut, float g, float& p,
                                           uint32_t& qm, uint32_t& qw, float um, float uw) {
  float m = 0.0f, v = 0.0f;
  if (!c.init) {
    const int q = (int)(int16_t)(uint16_t)qm;
    m = lut != nullptr ? decode_m_lut(q, lut) : decode_m(q, c.o_dm);
    v = decode_v(qw, c.o_wmin, c.o_dw, c.eps32);
  }
  float mn, vn;
  ema(c, g, m, v, mn, vn);
  p = adamw(c, p, mn, vn);
  qm = (uint32_t)(uint16_t)(int16_t)quant_m(c, mn, um);
  qw = quant_w(c, vn, uw);
}

// Raw bits of one pair of every stream, as loaded (fp32: two words, 16-bit
// types: one word).  Kept packed so the next pair can be prefetched while the
// current one is computed, at a few registers' cost.
struct RawPair {
  uint32_t p[2], g[2], qm, qw;
};

template <int DT>
__device__ __forceinline__ void raw2(const void* base, int64_t e, bool both, bool vec, uint32_t (&w)[2]) {
  if (DT == LUMA_F32) {
    const uint32_t* p = static_cast<const uint32_t*>(base) + e;
    if (vec) {
      const uint2 a = __ldcs(reinterpret_cast<const uint2*>(p));
      w[0] = a.x; w[1] = a.y;
    } else {
      w[0] = p[0]; w[1] = both ? p[1] : 0u;
    }
  } else {
    const uint16_t* p = static_cast<const uint16_t*>(base) + e;
    if (vec) {
      w[0] = __ldcs(reinterpret_cast<const unsigned int*>(p));
    } else {
      w[0] = (uint32_t)p[0] | (both ? (uint32_t)p[1] << 16 : 0u);
    }
  }
}

template <int DT>
__device__ __forceinline__ void unpack2(const uint32_t (&w)[2], float& x0, float& x1) {
  if (DT == LUMA_F32) {
    x0 = __uint_as_float(w[0]); x1 = __uint_as_float(w[1]);
  } else if (DT == LUMA_BF16) {
    x0 = __uint_as_float(w[0] << 16);  // bf16 -> f32 is exact
    x1 = __uint_as_float(w[0] & 0xFFFF0000u);
  } else {
    x0 = __half2float(__ushort_as_half((unsigned short)(w[0] & 0xFFFFu)));
    x1 = __half2float(__ushort_as_half((unsigned short)(w[0] >> 16)));
  }
}

template <int PD, int GD>
__device__ __forceinline__ void load_raw_pair(const LumaTensorDesc& d, bool init, bool vec2,
                                              int64_t P, RawPair& r) {
  const int64_t e = 2 * P;
  const bool both = e + 1 < d.numel;
  const bool vec = vec2 && both;
  raw2<PD>(d.param, e, both, vec, r.p);
  raw2<GD>(d.grad, e, both, vec, r.g);
  r.qm = 0u;
  r.qw = 0u;
  if (!init) {
    const uint16_t* qm = reinterpret_cast<const uint16_t*>(d.q_m) + e;
    const uint16_t* qw = reinterpret_cast<const uint16_t*>(d.q_w) + e;
    if (vec) {
      r.qm = __ldcs(reinterpret_cast<const unsigned int*>(qm));
      r.qw = __ldcs(reinterpret_cast<const unsigned int*>(qw));
    } else {
      r.qm = (uint32_t)qm[0] | (both ? (uint32_t)qm[1] << 16 : 0u);
      r.qw = (uint32_t)qw[0] | (both ? (uint32_t)qw[1] << 16 : 0u);
    }
  }
}

// Pass 2 over pairs [p_lo, p_hi) of a tensor, any alignment, injected or
// Philox uniforms, partial last pair: pair P holds elements 2P, 2P+1 and
// draws Philox block (rng_offset / 2 + P).  The steady state of aligned
// tensors runs in pass2_fast below.
template <int PD, int GD>
__device__ __forceinline__ void pass2_pairs(const LumaTensorDesc& d, const Consts& c,
                                            const float* lut, uint32_t k0, uint32_t k1, bool vec2,
                                            int64_t p_lo, int64_t p_hi) {
  constexpr int kThreads = kThreadsPass2;
  const bool injected = d.u_m != nullptr;
  const uint64_t ctr0 = (uint64_t)d.rng_offset >> 1;
  for (int64_t P = p_lo + threadIdx.x; P < p_hi; P += kThreads) {
    RawPair cur;
    load_raw_pair<PD, GD>(d, c.init, vec2, P, cur);
    const int64_t e = 2 * P;
    const bool both = e + 1 < d.numel;
    const bool vec = vec2 && both;
    float p0, p1, g0, g1;
    unpack2<PD>(cur.p, p0, p1);
    unpack2<GD>(cur.g, g0, g1);
    scale_grads2<GD>(c, g0, g1);
    uint32_t qm0 = cur.qm & 0xFFFFu, qm1 = cur.qm >> 16;
    uint32_t qw0 = cur.qw & 0xFFFFu, qw1 = cur.qw >> 16;
    float um0, um1, uw0, uw1;
    if (injected) {
      load2<LUMA_F32>(d.u_m, e, both, vec, um0, um1);
      load2<LUMA_F32>(d.u_w, e, both, vec, uw0, uw1);
      um0 *= kUScale; um1 *= kUScale; uw0 *= kUScale; uw1 *= kUScale;  // exact
    } else {
      const uint64_t ctr = ctr0 + (uint64_t)P;
      const uint4 r = philox4x32_10(make_uint4((uint32_t)ctr, (uint32_t)(ctr >> 32), 0u, 0u), k0, k1);
      um0 = u24_scaled(r.x); uw0 = u24_scaled(r.y); um1 = u24_scaled(r.z); uw1 = u24_scaled(r.w);
    }
    pass2_elem(c, lut, g0, p0, qm0, qw0, um0, uw0);
    pass2_elem(c, lut, g1, p1, qm1, qw1, um1, uw1);
    store_param2<PD>(d, e, both, vec, p0, p1);
    store2_codes(d.q_m, e, both, vec, qm0, qm1);
    store2_codes(d.q_w, e, both, vec, qw0, qw1);
  }
}

// Pass 2 over pairs [p_lo, p_hi) of a tensor, prefetching: pair P holds
// elements 2P, 2P+1 and draws Philox block (rng_offset / 2 + P); the next
// pair's loads are issued before the current pair is computed.  Used for bf16
// params, where it measured faster than pass2_fast.
template <int PD, int GD>
__device__ __forceinline__ void pass2_prefetch(const LumaTensorDesc& d, const Consts& c,
                                            const float* lut, uint32_t k0, uint32_t k1, bool vec2,
                                            int64_t p_lo, int64_t p_hi) {
  constexpr int kThreads = kThreadsPass2;
  const bool injected = d.u_m != nullptr;
  const uint64_t ctr0 = (uint64_t)d.rng_offset >> 1;
  int64_t P = p_lo + threadIdx.x;
  RawPair cur;
  if (P < p_hi) load_raw_pair<PD, GD>(d, c.init, vec2, P, cur);
  for (; P < p_hi; P += kThreads) {
    RawPair nxt;
    if (P + kThreads < p_hi) load_raw_pair<PD, GD>(d, c.init, vec2, P + kThreads, nxt);
    const int64_t e = 2 * P;
    const bool both = e + 1 < d.numel;
    const bool vec = vec2 && both;
    float p0, p1, g0, g1;
    unpack2<PD>(cur.p, p0, p1);
    unpack2<GD>(cur.g, g0, g1);
    scale_grads2<GD>(c, g0, g1);
    uint32_t qm0 = cur.qm & 0xFFFFu, qm1 = cur.qm >> 16;
    uint32_t qw0 = cur.qw & 0xFFFFu, qw1 = cur.qw >> 16;
    float um0, um1, uw0, uw1;
    if (injected) {
      load2<LUMA_F32>(d.u_m, e, both, vec, um0, um1);
      load2<LUMA_F32>(d.u_w, e, both, vec, uw0, uw1);
      um0 *= kUScale; um1 *= kUScale; uw0 *= kUScale; uw1 *= kUScale;  // exact
    } else {
      const uint64_t ctr = ctr0 + (uint64_t)P;
      const uint4 r = philox4x32_10(make_uint4((uint32_t)ctr, (uint32_t)(ctr >> 32), 0u, 0u), k0, k1);
      um0 = u24_scaled(r.x); uw0 = u24_scaled(r.y); um1 = u24_scaled(r.z); uw1 = u24_scaled(r.w);
    }
    pass2_elem(c, lut, g0, p0, qm0, qw0, um0, uw0);
    pass2_elem(c, lut, g1, p1, qm1, qw1, um1, uw1);
    store_param2<PD>(d, e, both, vec, p0, p1);
    store2_codes(d.q_m, e, both, vec, qm0, qm1);
    store2_codes(d.q_w, e, both, vec, qw0, qw1);
    cur = nxt;
  }
}

// Steady-state pass 2 over n complete, 16-byte-aligned pairs with Philox
// uniforms: pair-typed pointers to the first pair, 32-bit indices, no
// per-pair tail or alignment tests.  Same arithmetic as pass2_pairs.
template <int DT>
struct PairWord {  // one pair of a stream as a single load/store unit
  using T = typename std::conditional<DT == LUMA_F32, uint2, uint32_t>::type;
};

template <int DT>
__device__ __forceinline__ void to_words(const typename PairWord<DT>::T& v, uint32_t (&w)[2]) {
  if constexpr (DT == LUMA_F32) { w[0] = v.x; w[1] = v.y; } else { w[0] = v; w[1] = 0u; }
}

template <int PD, int GD>
__device__ __forceinline__ void pass2_fast(const Consts& c, const float* lut, uint32_t k0,
                                           uint32_t k1, typename PairWord<PD>::T* mcp,
                                           bool mc_local, typename PairWord<PD>::T* pp,
                                           const typename PairWord<GD>::T* gp, uint32_t* qmp,
                                           uint32_t* qwp, uint64_t ctr_base, int n) {
  constexpr int kThreads = kThreadsPass2;
  int i = threadIdx.x;
  RawPair cur;
  auto load = [&](int j, RawPair& r) {
    to_words<PD>(__ldcs(pp + j), r.p);
    to_words<GD>(__ldcs(gp + j), r.g);
    r.qm = c.init ? 0u : __ldcs(qmp + j);
    r.qw = c.init ? 0u : __ldcs(qwp + j);
  };
  if (i < n) load(i, cur);
  for (; i < n; i += kThreads) {
    RawPair nxt;
    if (i + kThreads < n) load(i + kThreads, nxt);
    float p0, p1, g0, g1;
    unpack2<PD>(cur.p, p0, p1);
    unpack2<GD>(cur.g, g0, g1);
    scale_grads2<GD>(c, g0, g1);
    uint32_t qm0 = cur.qm & 0xFFFFu, qm1 = cur.qm >> 16;
    uint32_t qw0 = cur.qw & 0xFFFFu, qw1 = cur.qw >> 16;
    const uint64_t ctr = ctr_base + (uint32_t)i;
    const uint4 r = philox4x32_10(make_uint4((uint32_t)ctr, (uint32_t)(ctr >> 32), 0u, 0u), k0, k1);
    const float um0 = u24_scaled(r.x), uw0 = u24_scaled(r.y);
    const float um1 = u24_scaled(r.z), uw1 = u24_scaled(r.w);
    pass2_elem(c, lut, g0, p0, qm0, qw0, um0, uw0);
    pass2_elem(c, lut, g1, p1, qm1, qw1, um1, uw1);
    if (mcp != nullptr) mc_store2<PD>(mcp, 2 * (int64_t)i, true, p0, p1);
    if (mcp == nullptr || mc_local) {
      if constexpr (PD == LUMA_F32) {
        __stcs(pp + i, make_uint2(__float_as_uint(p0), __float_as_uint(p1)));
      } else {
        __stcs(pp + i, (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(p0)) |
                           ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(p1)) << 16));
      }
    }
    __stcs(qmp + i, (qm0 & 0xFFFFu) | (qm1 << 16));
    __stcs(qwp + i, (qw0 & 0xFFFFu) | (qw1 << 16));
    cur = nxt;
  }
}

// ---------------------------------------------------------------------------
// Steady-state pass 2: step >= 2 with the decode table, Philox uniforms,
// aligned complete pairs, and a segment whose grids keep every operand of the
// correctly rounded arithmetic above inside its verified range (hot_segment).
// The arithmetic is that of pass2_elem with two differences that leave the
// results unchanged: rcp_cr / sqrt_cr / div_cr replace the IEEE intrinsics,
// and each LogSR decision is taken from the series value alone.  An element
// whose m' or v' falls outside the verified range (tiny, subnormal or NaN), or
// whose decision would need expm1f (u within the margin of the series value,
// about 4e-6 of the decisions), marks its pair; a marked pair is recomputed by
// pass2_pair_exact with the general code, which also stores it.
// ---------------------------------------------------------------------------

// Bounds of the verified ranges, with margin (see rcp_cr / sqrt_cr / div_cr).
constexpr float kHotMinV = 0x1.0p-100f;   // v' (and v'/bc2 >= v'): sqrt_cr
constexpr float kHotMinM = 0x1.0p-80f;    // |m'|: quotient >= 2^-120 when den <= 2^40
constexpr double kHotMaxDen = 0x1.0p40;   // sqrt(S_v / bc2) + eps
constexpr double kHotMaxQuot = 0x1.0p119; // S_m / eps
constexpr double kHotMaxM = 0x1.0p100;
constexpr double kHotMinEps = 0x1.0p-100;
constexpr double kHotMinW = 0x1.0p-124;   // decode w range: rcp_cr
constexpr double kHotMaxW = 0x1.0p123;

// Whether every element of the segment satisfies the range conditions that do
// not depend on the element: eps, the decode grid's w range, and the maxima
// S_m / S_v of this step bounding |m'|, v', the AdamW denominator and quotient.
__device__ __forceinline__ bool hot_segment(const SegShared& s) {
  const double eps = (double)s.row.eps32;
  const double w_lo = (double)s.dec.w_min;
  const double w_hi = w_lo * exp(65535.0 * (double)s.dec.dw) * 2.0;  // decode w <= this
  const double den_hi = sqrt(s.enc.S_v * (double)s.row.inv_bc2 * 2.0) + eps * 2.0;
  return eps >= kHotMinEps && w_lo >= kHotMinW && w_hi <= kHotMaxW &&
         s.enc.S_m <= kHotMaxM && s.enc.S_m <= kHotMaxQuot * eps && den_hi <= kHotMaxDen;
}

// Float to 16-bit integer conversions, truncating (the arguments are integral)
// and saturating to the destination range (PTX cvt clamps float-to-integer
// results); the result's 16 bits in the low half of a 32-bit word.
__device__ __forceinline__ uint32_t f2u16_sat(float x) {
  unsigned short h;
  asm("cvt.rzi.u16.f32 %0, %1;" : "=h"(h) : "f"(x));
  return (uint32_t)h;
}

__device__ __forceinline__ uint32_t f2i16_bits(float x) {
  unsigned short h;
  asm("cvt.rzi.s16.f32 %0, %1;" : "=h"(h) : "f"(x));
  return (uint32_t)h;
}

// Two floats rounded to bf16 (RN) and packed, the first in the low half.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  uint32_t u;
  memcpy(&u, &h, sizeof(u));
  return u;
}

// pass2_elem for the steady state; sets `rare` when the element's results may
// differ from pass2_elem's (they are then discarded).  Every value of an
// element that is not marked is finite, so the NaN-keeping clamps of the
// general code become plain fminf / fmaxf here.
__device__ __forceinline__ void pass2_elem_hot(const Consts& c, const float* lut, float g, float& p,
                                               uint32_t& qm, uint32_t& qw, float um, float uw,
                                               bool& rare) {
  const float m = decode_m_lut((int)(int16_t)(uint16_t)qm, lut);
  float t = __fsub_rn(rcp_cr(__fmul_rn(c.o_wmin, expf(__fmul_rn((float)qw, c.o_dw)))), c.eps32);
  t = fmaxf(t, 0.0f);
  const float v = __fmul_rn(t, t);
  const float mn = __fadd_rn(__fmul_rn(c.beta1, m), __fmul_rn(c.omb1, g));
  const float vn = __fadd_rn(__fmul_rn(c.beta2, v), __fmul_rn(c.omb2, __fmul_rn(g, g)));
  // v' = +0 takes sqrt = +0; m' = +0 gives the quotient +0 (div_cr(+0, den) = +0).
  const bool v_ok = vn >= kHotMinV;
  const bool v_zero = __float_as_uint(vn) == 0u;
  rare |= !(v_ok || v_zero) || !(fabsf(mn) >= kHotMinM || __float_as_uint(mn) == 0u);
  {  // AdamW
    const float pd = __fmul_rn(p, c.decay);
    const float sq = v_ok ? sqrt_cr(__fmul_rn(vn, c.inv_bc2)) : 0.0f;
    p = __fmaf_rn(c.neg_eta, div_cr(mn, __fadd_rn(sq, c.eps32)), pd);
  }
  {  // quant_m
    const float a = fabsf(mn);
    const float ac = fminf(a, c.n_sm32);
    const float y = __fmul_rn(log1pf(ac), c.n_inv_dm);
    const float fy = floorf(y);
    const float fr = __fsub_rn(y, fy);  // exact
    const float diff =
        __fmaf_rn(-fr, __fmaf_rn(fr, __fmaf_rn(fr, g_seg.pm3, g_seg.pm2), g_seg.pm1), um);
    rare |= !(fabsf(diff) > kHotMargin);
    // y >= 0, so r >= 0; the sign of m' goes onto r and the conversion is exact
    const float r = fminf(__fadd_rn(fy, diff < 0.0f ? 1.0f : 0.0f), (float)LUMA_K_M);
    qm = f2i16_bits(__uint_as_float(__float_as_uint(r) | (__float_as_uint(mn) & 0x80000000u)));
  }
  {  // quant_w
    const float sq = v_ok ? sqrt_cr(vn) : 0.0f;
    const float w = fminf(fmaxf(rcp_cr(__fadd_rn(sq, c.eps32)), c.n_wmin), c.w_max);
    const float y = __fmul_rn(logf(__fmul_rn(w, c.n_inv_wmin)), c.n_inv_dw);
    const float fy = floorf(y);
    const float fr = __fsub_rn(y, fy);  // exact
    const float diff =
        __fmaf_rn(-fr, __fmaf_rn(fr, __fmaf_rn(fr, g_seg.pw3, g_seg.pw2), g_seg.pw1), uw);
    rare |= !(fabsf(diff) > kHotMargin);
    // clamp(0, K_W = 65535) is the saturation of the conversion to u16
    qw = f2u16_sat(__fadd_rn(fy, diff < 0.0f ? 1.0f : 0.0f));
  }
}

// A marked pair (element index e = 2P, both elements present, aligned):
// reload, recompute with pass2_elem and store.  Out of line so the steady
// loop's registers are not shaped by this rarely run code.
template <int PD, int GD>
__device__ __noinline__ void pass2_pair_exact(uint32_t k0, uint32_t k1, int64_t P) {
  const LumaTensorDesc& d = g_seg.d;
  const float* lut = g_lut;
  Consts c;
  fill_consts(g_seg, true, c);
  RawPair r;
  load_raw_pair<PD, GD>(d, false, true, P, r);
  float p0, p1, g0, g1;
  unpack2<PD>(r.p, p0, p1);
  unpack2<GD>(r.g, g0, g1);
  scale_grads2<GD>(c, g0, g1);
  uint32_t qm0 = r.qm & 0xFFFFu, qm1 = r.qm >> 16;
  uint32_t qw0 = r.qw & 0xFFFFu, qw1 = r.qw >> 16;
  const uint64_t ctr = ((uint64_t)d.rng_offset >> 1) + (uint64_t)P;
  const uint4 u = philox4x32_10(make_uint4((uint32_t)ctr, (uint32_t)(ctr >> 32), 0u, 0u), k0, k1);
  pass2_elem(c, lut, g0, p0, qm0, qw0, u24_scaled(u.x), u24_scaled(u.y));
  pass2_elem(c, lut, g1, p1, qm1, qw1, u24_scaled(u.z), u24_scaled(u.w));
  const int64_t e = 2 * P;
  store_param2<PD>(d, e, true, true, p0, p1);
  store2_codes(d.q_m, e, true, true, qm0, qm1);
  store2_codes(d.q_w, e, true, true, qw0, qw1);
}

// The steady loop over n complete pairs starting at pair p_lo of the segment.
// Each thread takes pairs i and i + kThreads of every block of 2 * kThreads
// (both coalesced across the warp): one interleaved Philox evaluation for the
// two, two independent element chains each, and the copies of the next
// kHotStages / 2 - 1 iterations in flight.  Measured on one Llama-3-8B layer
// (bf16): 512 threads x 2 pairs 1.80 ms with copies 1 iteration ahead, 1.82 ms
// 2 iterations ahead; 640 x 1 pair 1.89 ms, 640 x 2 pairs 1.96 ms (register
// spills), 448 x 2 pairs 2.07 ms.
template <int PD, int GD>
__device__ __forceinline__ void pass2_hot(const SegShared& s, const Consts& c, const float* lut,
                                           uint32_t k0, uint32_t k1, int64_t p_lo, int n) {
  constexpr int kThreads = kThreadsPass2;
  constexpr int kS = kHotStages / 2;
  using PW = typename PairWord<PD>::T;
  using GW = typename PairWord<GD>::T;
  const LumaTensorDesc& d = s.d;
  PW* pp = static_cast<PW*>(d.param) + p_lo;
  PW* mcp = d.param_mc != nullptr ? static_cast<PW*>(d.param_mc) + p_lo : nullptr;
  const GW* gp = static_cast<const GW*>(d.grad) + p_lo;
  uint32_t* qmp = reinterpret_cast<uint32_t*>(d.q_m) + p_lo;
  uint32_t* qwp = reinterpret_cast<uint32_t*>(d.q_w) + p_lo;
  const uint64_t ctr_base = ((uint64_t)d.rng_offset >> 1) + (uint64_t)p_lo;
  unsigned char* stage0 = reinterpret_cast<unsigned char*>(g_lut) + kLutPadBytes;
  PW* sp = reinterpret_cast<PW*>(stage0) + threadIdx.x;
  GW* sg = reinterpret_cast<GW*>(stage0 + (size_t)kThreadsPass2 * 8) + threadIdx.x;
  uint32_t* sm = reinterpret_cast<uint32_t*>(stage0 + (size_t)kThreadsPass2 * 16) + threadIdx.x;
  uint32_t* sw = reinterpret_cast<uint32_t*>(stage0 + (size_t)kThreadsPass2 * 20) + threadIdx.x;
  constexpr int kStageWords = (int)(kHotStageBytes / 4);
  auto issue = [&](int j, int st) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int jj = j + h * kThreads;
      if (jj < n) {
        const int o = (2 * st + h) * kStageWords;
        cp_async<sizeof(PW)>(reinterpret_cast<uint32_t*>(sp) + o, pp + jj);
        cp_async<sizeof(GW)>(reinterpret_cast<uint32_t*>(sg) + o, gp + jj);
        cp_async<4>(sm + o, qmp + jj);
        cp_async<4>(sw + o, qwp + jj);
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int k = 0; k < kS - 1; ++k) issue(threadIdx.x + k * 2 * kThreads, k);
  int st = 0;
  for (int i = threadIdx.x; i < n; i += 2 * kThreads) {
    issue(i + (kS - 1) * 2 * kThreads, st == 0 ? kS - 1 : st - 1);
    cp_async_wait<kS - 1>();
    const int o0 = (2 * st) * kStageWords, o1 = o0 + kStageWords;
    RawPair cur0, cur1;
    to_words<PD>(*reinterpret_cast<const PW*>(reinterpret_cast<const uint32_t*>(sp) + o0), cur0.p);
    to_words<GD>(*reinterpret_cast<const GW*>(reinterpret_cast<const uint32_t*>(sg) + o0), cur0.g);
    cur0.qm = sm[o0];
    cur0.qw = sw[o0];
    to_words<PD>(*reinterpret_cast<const PW*>(reinterpret_cast<const uint32_t*>(sp) + o1), cur1.p);
    to_words<GD>(*reinterpret_cast<const GW*>(reinterpret_cast<const uint32_t*>(sg) + o1), cur1.g);
    cur1.qm = sm[o1];
    cur1.qw = sw[o1];
    st = st == kS - 1 ? 0 : st + 1;
    const bool has1 = i + kThreads < n;
    const uint64_t ca = ctr_base + (uint32_t)i, cb = ca + kThreads;
    uint4 ra = make_uint4((uint32_t)ca, (uint32_t)(ca >> 32), 0u, 0u);
    uint4 rb = make_uint4((uint32_t)cb, (uint32_t)(cb >> 32), 0u, 0u);
    philox_x2(ra, rb, k0, k1);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (h == 1 && !has1) break;
      const RawPair& cur = h == 0 ? cur0 : cur1;
      const uint4& r = h == 0 ? ra : rb;
      const int ii = i + h * kThreads;
      float p0, p1, g0, g1;
      unpack2<PD>(cur.p, p0, p1);
      unpack2<GD>(cur.g, g0, g1);
      scale_grads2<GD>(c, g0, g1);
      uint32_t qm0 = cur.qm & 0xFFFFu, qm1 = cur.qm >> 16;
      uint32_t qw0 = cur.qw & 0xFFFFu, qw1 = cur.qw >> 16;
      bool rare = false;
      pass2_elem_hot(c, lut, g0, p0, qm0, qw0, u24_scaled(r.x), u24_scaled(r.y), rare);
      pass2_elem_hot(c, lut, g1, p1, qm1, qw1, u24_scaled(r.z), u24_scaled(r.w), rare);
      if (rare) {
        pass2_pair_exact<PD, GD>(k0, k1, p_lo + ii);
      } else {
        // the multicast mapping (replica: it includes this GPU's copy), and
        // the param itself unless the mapping covers it
        if (mcp != nullptr) mc_store2<PD>(mcp, 2 * (int64_t)ii, true, p0, p1);
        if (mcp == nullptr || d.mc_local) {
          if constexpr (PD == LUMA_F32) {
            __stcs(pp + ii, make_uint2(__float_as_uint(p0), __float_as_uint(p1)));
          } else {
            __stcs(pp + ii, pack_bf16x2(p0, p1));
          }
        }
        __stcs(qmp + ii, __byte_perm(qm0, qm1, 0x5410));
        __stcs(qwp + ii, __byte_perm(qw0, qw1, 0x5410));
      }
    }
  }
  cp_async_wait<0>();
}

// Pass 2 for one tensor segment.  bf16 params: the prefetching pair loop.
// fp32 params: the steady-state loop where it applies, the general loop
// otherwise (unaligned views, injected uniforms, the odd tail).  The choice
// per param dtype is measured (one Llama-3-8B layer and GPT-2 small).
template <int PD, int GD>
__device__ __forceinline__ void pass2_segment(const SegShared& s, const Consts& c,
                                              const float* lut, uint32_t k0, uint32_t k1,
                                              bool vec2, int64_t p_lo, int64_t p_hi) {
  const LumaTensorDesc& d = s.d;
  const int64_t p_full = min(p_hi, d.numel / 2);  // pairs with both elements
  const bool steady = vec2 && d.u_m == nullptr && p_full > p_lo && p_full - p_lo <= 0x7FFFFFFF;
  if (steady && !c.init && lut != nullptr && hot_segment(s)) {
    pass2_hot<PD, GD>(s, c, lut, k0, k1, p_lo, (int)(p_full - p_lo));
    if (p_full < p_hi) pass2_pairs<PD, GD>(d, c, lut, k0, k1, vec2, p_full, p_hi);
    return;
  }
  if constexpr (PD == LUMA_BF16) {
    pass2_prefetch<PD, GD>(d, c, lut, k0, k1, vec2, p_lo, p_hi);
    return;
  }
  if (steady) {
    using PW = typename PairWord<PD>::T;
    using GW = typename PairWord<GD>::T;
    pass2_fast<PD, GD>(c, lut, k0, k1,
                       d.param_mc != nullptr ? static_cast<PW*>(d.param_mc) + p_lo : nullptr,
                       d.mc_local != 0, static_cast<PW*>(d.param) + p_lo,
                       static_cast<const GW*>(d.grad) + p_lo,
                       reinterpret_cast<uint32_t*>(d.q_m) + p_lo,
                       reinterpret_cast<uint32_t*>(d.q_w) + p_lo,
                       ((uint64_t)d.rng_offset >> 1) + (uint64_t)p_lo, (int)(p_full - p_lo));
    if (p_full < p_hi) pass2_pairs<PD, GD>(d, c, lut, k0, k1, vec2, p_full, p_hi);
  } else {
    pass2_pairs<PD, GD>(d, c, lut, k0, k1, vec2, p_lo, p_hi);
  }
}

// ---------------------------------------------------------------------------
// Kernels
// ---------------------------------------------------------------------------

// One tensor segment of pass 2 for one (param, grad) dtype pair, the step
// constants read from the segment state in shared memory.  (Inlined: an
// out-of-line version per dtype pair measured 3% slower.)
template <int PD, int GD>
__device__ __forceinline__ void pass2_segment_from_shared(bool use_lut, uint32_t k0, uint32_t k1, bool vec2,
                                              int64_t p_lo, int64_t p_hi) {
  Consts c;
  fill_consts(g_seg, true, c);
  pass2_segment<PD, GD>(g_seg, c, use_lut ? g_lut : nullptr, k0, k1, vec2, p_lo, p_hi);
}

// Segment-level selection of the pass-2 loop for the tensor's dtypes.
__device__ __forceinline__ void dispatch_pass2(const SegShared& s, const float* lut, uint32_t k0,
                                               uint32_t k1, bool vec2, int64_t p_lo,
                                               int64_t p_hi) {
  const LumaTensorDesc& d = s.d;
  if (d.param_dtype == LUMA_F32) {
    switch (d.grad_dtype) {
      case LUMA_F32: pass2_segment_from_shared<LUMA_F32, LUMA_F32>(lut != nullptr, k0, k1, vec2, p_lo, p_hi); break;
      case LUMA_BF16: pass2_segment_from_shared<LUMA_F32, LUMA_BF16>(lut != nullptr, k0, k1, vec2, p_lo, p_hi); break;
      default: pass2_segment_from_shared<LUMA_F32, LUMA_F16>(lut != nullptr, k0, k1, vec2, p_lo, p_hi); break;
    }
  } else {
    switch (d.grad_dtype) {
      case LUMA_F32: pass2_segment_from_shared<LUMA_BF16, LUMA_F32>(lut != nullptr, k0, k1, vec2, p_lo, p_hi); break;
      case LUMA_BF16: pass2_segment_from_shared<LUMA_BF16, LUMA_BF16>(lut != nullptr, k0, k1, vec2, p_lo, p_hi); break;
      default: pass2_segment_from_shared<LUMA_BF16, LUMA_F16>(lut != nullptr, k0, k1, vec2, p_lo, p_hi); break;
    }
  }
}

// Largest i with descs[i].oct_begin <= pos.
__device__ int find_desc(const LumaTensorDesc* descs, int n, int64_t pos) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (descs[mid].oct_begin <= pos) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Thread 0: load descriptor `di`, its row and grids into shared memory.
__device__ void load_segment(const LumaStepArgs& a, int di, bool pass2, SegShared& s) {
  s.d = a.descs[di];
  s.skip = 0;
  s.has_gscale = a.grad_scale != nullptr;
  s.gscale = a.grad_scale != nullptr ? *a.grad_scale : 1.0f;
  s.check_inf = a.found_inf != nullptr;
  if (a.step_counters != nullptr) {
    // Capturable mode: the step count lives on the device; the row of step t
    // is entry t - 1 of the descriptor's block of the row table.
    const int64_t t = a.step_counters[s.d.slot] + 1;
    const int64_t r = (int64_t)s.d.row + t - 1;
    if (t < 1 || r >= (int64_t)a.n_rows) {
      s.skip = 1;
      atomicOr(&g_kernel_error, (unsigned int)LUMA_KERR_ROW_RANGE);
      return;
    }
    s.row = a.rows[r];
  } else {
    s.row = a.rows[s.d.row];
  }
  const LumaSlot* slot = a.slots + s.d.slot;
  const int64_t t = s.row.step;
  if (t != 1) {
    s.dec = slot->grid[(t - 1) & 1];
    // The stored grid was derived with the eps of its own step; the reference
    // re-derives the decode grid from (S_m, S_v) with the current eps.
    if (s.dec.eps != s.row.eps) make_grid(s.dec.S_m, s.dec.S_v, s.row.eps, &s.dec);
  }
  if (pass2) {
    s.enc = slot->grid[t & 1];
    series_coefs(s.enc.dm, s.enc.inv_zm, s.pm1, s.pm2, s.pm3);
    series_coefs(s.enc.dw, s.enc.inv_zw, s.pw1, s.pw2, s.pw3);
  }
}

// kStaticAcc: pass-1 accumulators at acc[descriptor index] (luma_step_noalloc)
// instead of in the caller's LumaSlot (luma_step).
template <bool PASS2, bool kStaticAcc = false>
__global__ void __launch_bounds__(PASS2 ? kThreadsPass2 : kThreadsPass1, 1)
luma_pass_kernel(const LumaStepArgs a, const int lut_ok, PassAccum* acc) {
  constexpr int kThreads = PASS2 ? kThreadsPass2 : kThreadsPass1;
  constexpr int kWarps = kThreads / 32;
  SegShared& s = g_seg;
  __shared__ uint32_t red_m[kMaxWarps], red_v[kMaxWarps];
  __shared__ float s_vbound[256];  // pass 1: bucket maxima of the decoded v
  __shared__ int s_di;
  float* s_lut = g_lut;

  const int64_t T = a.total_octets;
  const int64_t lo = (T * (int64_t)blockIdx.x) / (int64_t)gridDim.x;
  const int64_t hi = (T * ((int64_t)blockIdx.x + 1)) / (int64_t)gridDim.x;
  if (lo >= hi) return;
  // A non-finite grad seen by pass 1 (or flagged by the caller before the
  // step) skips the update of every tensor, as GradScaler.step skips
  // optimizer.step().  Pass 1 has already finished: same stream.
  if (PASS2 && a.found_inf != nullptr && *a.found_inf != 0.0f) return;

  if (threadIdx.x == 0) s_di = find_desc(a.descs, a.n_desc, lo);
  __syncthreads();
  int di = s_di;
  int64_t pos = lo;
  while (pos < hi && di < a.n_desc) {
    if (threadIdx.x == 0) load_segment(a, di, PASS2, s);
    __syncthreads();
    const LumaTensorDesc& d = s.d;
    const int64_t n_oct = (d.numel + 7) / 8;
    const int64_t o_lo = pos - d.oct_begin;
    const int64_t o_hi = min(hi - d.oct_begin, n_oct);
    if (s.skip) {  // (uniform) no row for this step: leave the tensor as it is
      __syncthreads();
      pos = d.oct_begin + o_hi;
      ++di;
      continue;
    }
    Consts c;
    fill_consts(s, PASS2, c);
    // Decode table for long segments of quantized (t >= 2) tensors; in pass
    // 1 also the bucket maxima of v(q) (256 buckets of 256 codes): thread i
    // evaluates codes [c i, c i + c) with c = 65536 / threads, and the
    // 256 / c consecutive lanes of a bucket combine their maxima.
    const float* lut = nullptr;
    const float* vbt = nullptr;
    bool qb = false;  // pass 1: quad bounds usable (quad_may_raise)
    if (lut_ok && !c.init && (o_hi - o_lo) * 8 >= kLutMinElems) {
      for (int i = threadIdx.x; i < kLutEntries; i += kThreads)
        s_lut[i] = expm1f(__fmul_rn((float)i, c.o_dm));
      if (!PASS2) {
        constexpr int kCodes = 65536 / kThreads;     // codes per thread
        constexpr int kLanes = 256 / kCodes;         // lanes per bucket
        static_assert(PASS2 || (kCodes * kThreads == 65536 && kLanes >= 1 && kLanes <= 32),
                      "bucket table layout");
        uint32_t mx = 0u;
        for (int j = 0; j < kCodes; ++j)
          mx = max(mx, __float_as_uint(decode_v((uint32_t)(threadIdx.x * kCodes + j), c.o_wmin,
                                                c.o_dw, c.eps32)));
#pragma unroll
        for (int k = 1; k < kLanes; k <<= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, k));
        if (threadIdx.x % kLanes == 0) s_vbound[threadIdx.x / kLanes] = __uint_as_float(mx);
        vbt = s_vbound;
      }
      __syncthreads();
      lut = s_lut;
      if (!PASS2) {
        // Quad bounds need vbt non-increasing and lut non-decreasing.  vbt
        // becomes its suffix maxima (still >= v(q) of every code of a bucket;
        // v(q) falls with q, so this loosens it little), warp 0, eight entries
        // per lane.  lut, the exact decode table, is only checked: one
        // inversion (not seen, the entries are spaced by a factor >= e^dm)
        // or a NaN entry turns the quad bounds off for the segment.
        if (threadIdx.x < 32) {
          uint32_t e[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) e[k] = __float_as_uint(s_vbound[threadIdx.x * 8 + k]);
#pragma unroll
          for (int k = 6; k >= 0; --k) e[k] = max(e[k], e[k + 1]);
          uint32_t sfx = e[0];  // suffix maximum over lanes >= this one
#pragma unroll
          for (int k = 1; k < 32; k <<= 1) {
            const uint32_t t = __shfl_down_sync(0xffffffffu, sfx, k);
            if (threadIdx.x + k < 32) sfx = max(sfx, t);
          }
          uint32_t nxt = __shfl_down_sync(0xffffffffu, sfx, 1);
          if (threadIdx.x == 31) nxt = 0u;
#pragma unroll
          for (int k = 0; k < 8; ++k) s_vbound[threadIdx.x * 8 + k] = __uint_as_float(max(e[k], nxt));
        }
        int inv = 0;
        for (int i = threadIdx.x; i < kLutEntries - 1; i += kThreads)
          inv |= !(s_lut[i] <= s_lut[i + 1]);
        qb = __syncthreads_or(inv) == 0;  // also publishes the suffix maxima
      }
    }

    if (!PASS2) {
      MaxSearch ms;
      // Staged loop for the complete octets of aligned tensors at step >= 2
      // (the staging area exists whenever the kernel has its shared memory,
      // i.e. lut_ok); plain loads for the rest.
      int64_t ob = o_lo;
      if (lut_ok && !c.init && d.vec_ok != 0) {
        const int64_t o_full = min(o_hi, d.numel / 8);
        if (o_full > o_lo) {
          switch (d.grad_dtype) {
            case LUMA_F32: pass1_staged<LUMA_F32>(d, c, lut, vbt, qb, 2 * o_lo, 2 * o_full, ms); break;
            case LUMA_BF16: pass1_staged<LUMA_BF16>(d, c, lut, vbt, qb, 2 * o_lo, 2 * o_full, ms); break;
            default: pass1_staged<LUMA_F16>(d, c, lut, vbt, qb, 2 * o_lo, 2 * o_full, ms); break;
          }
          ob = o_full;
        }
      }
      if (ob < o_hi) {
        switch (d.grad_dtype) {
          case LUMA_F32: pass1_octets<LUMA_F32>(d, c, lut, vbt, ob, o_hi, ms); break;
          case LUMA_BF16: pass1_octets<LUMA_BF16>(d, c, lut, vbt, ob, o_hi, ms); break;
          default: pass1_octets<LUMA_F16>(d, c, lut, vbt, ob, o_hi, ms); break;
        }
      }
      if (c.check_inf) {  // (uniform) any inf / NaN grad in this CTA's part
        if (__syncthreads_or(ms.bad) && threadIdx.x == 0) *a.found_inf = 1.0f;
      }
      uint32_t am = ms.am, av = ms.av;
      am = __reduce_max_sync(0xffffffffu, am);
      av = __reduce_max_sync(0xffffffffu, av);
      const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
      if (lane == 0) { red_m[warp] = am; red_v[warp] = av; }
      __syncthreads();
      if (threadIdx.x == 0) {
        for (int w = 1; w < kWarps; ++w) { am = max(am, red_m[w]); av = max(av, red_v[w]); }
        LumaSlot* slot = a.slots + d.slot;
        uint32_t* amax_m = kStaticAcc ? &acc[di].amax_m : &slot->amax_m;
        uint32_t* amax_v = kStaticAcc ? &acc[di].amax_v : &slot->amax_v;
        unsigned long long* done =
            kStaticAcc ? &acc[di].done : reinterpret_cast<unsigned long long*>(&slot->done);
        atomicMax(amax_m, am);
        atomicMax(amax_v, av);
        __threadfence();
        const unsigned long long mine = (unsigned long long)(o_hi - o_lo);
        const unsigned long long prev = atomicAdd(done, mine);
        if (prev + mine == (unsigned long long)n_oct) {
          // Last contributor for this tensor: every other CTA's maxima are in.
          __threadfence();
          const uint32_t bm = atomicOr(amax_m, 0u);
          const uint32_t bv = atomicOr(amax_v, 0u);
          const double smt = (double)__uint_as_float(bm);
          const double svt = (double)__uint_as_float(bv);
          // S_m = max(S_m_t, 1e-9); S_v = max(S_v_t, 0.0) with Python's max()
          // (first argument kept unless the second compares greater).
          const double S_m = (LUMA_SCALE_FLOOR_M > smt) ? LUMA_SCALE_FLOOR_M : smt;
          const double S_v = (0.0 > svt) ? 0.0 : svt;
          make_grid(S_m, S_v, s.row.eps, &slot->grid[s.row.step & 1]);
          *amax_m = 0u;
          *amax_v = 0u;
          *done = 0ull;
        }
      }
    } else {
      const uint64_t seed = ((uint64_t)s.row.step << 32 | (uint64_t)((int64_t)d.param_id * 2)) ^
                            (uint64_t)a.base_seed;
      const uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
      const int64_t n_pairs = (d.numel + 1) / 2;
      const int64_t p_lo = 4 * o_lo;
      const int64_t p_hi = min(4 * o_hi, n_pairs);
      const int pes = d.param_dtype == LUMA_F32 ? 8 : 4;   // bytes of a param pair
      const int ges = d.grad_dtype == LUMA_F32 ? 8 : 4;
      const bool vec2 = ((uintptr_t)d.param % pes == 0) && ((uintptr_t)d.grad % ges == 0) &&
                        ((uintptr_t)d.q_m % 4 == 0) && ((uintptr_t)d.q_w % 4 == 0) &&
                        ((uintptr_t)d.u_m % 8 == 0) && ((uintptr_t)d.u_w % 8 == 0);
      dispatch_pass2(s, lut, k0, k1, vec2, p_lo, p_hi);
      // multicast stores become visible on the peers before anything the
      // caller orders after the step (its cross-GPU barrier)
      if (d.param_mc != nullptr) __threadfence_system();
    }
    __syncthreads();  // s is rewritten for the next tensor
    pos = d.oct_begin + o_hi;
    ++di;
  }
}

// Capturable mode: the step count of every descriptor's slot advances by one
// after pass 2 (each slot appears in at most one descriptor of a call).
__global__ void __launch_bounds__(kThreads) luma_count_steps_kernel(const LumaTensorDesc* descs,
                                                                   int n, int64_t* counters,
                                                                   const float* found_inf) {
  if (found_inf != nullptr && *found_inf != 0.0f) return;  // skipped step
  const int i = blockIdx.x * kThreads + threadIdx.x;
  if (i < n) counters[descs[i].slot] += 1;
}

__global__ void __launch_bounds__(kThreads) luma_decode_kernel(
    const int16_t* __restrict__ q_m, const int16_t* __restrict__ q_w, int64_t n,
    float dm, float wmin, float dw, float eps32, float* __restrict__ m_out,
    float* __restrict__ v_out) {
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kThreads) {
    m_out[i] = decode_m((int)q_m[i], dm);
    v_out[i] = decode_v((uint32_t)(uint16_t)q_w[i], wmin, dw, eps32);
  }
}

// Self-check of rcp_cr / sqrt_cr / div_cr against the IEEE intrinsics on
// random operands drawn over their verified ranges (see rcp_cr).
__device__ unsigned long long g_arith_bad[3];

__device__ __forceinline__ uint64_t mix64(uint64_t x) {  // splitmix64 finaliser
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

__global__ void __launch_bounds__(kThreads) luma_arith_check_kernel(uint64_t n, uint64_t seed) {
  unsigned int bad[3] = {0u, 0u, 0u};
  for (uint64_t i = (uint64_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * kThreads) {
    const uint64_t h = mix64(seed ^ mix64(i));
    const uint64_t h2 = mix64(h);
    // rcp: |b| in [2^-125, 2^125): biased exponent 2..251, any significand and sign
    const float b = __uint_as_float((uint32_t)(h >> 63) << 31 |
                                    (uint32_t)(2 + (h >> 32) % 250) << 23 | ((uint32_t)h & 0x7FFFFFu));
    bad[0] += __float_as_uint(rcp_cr(b)) != __float_as_uint(__frcp_rn(b));
    // sqrt: x in [2^-102, FLT_MAX]: biased exponent 25..254
    const float x = __uint_as_float((uint32_t)(25 + (h2 >> 32) % 230) << 23 | ((uint32_t)h2 & 0x7FFFFFu));
    bad[1] += __float_as_uint(sqrt_cr(x)) != __float_as_uint(__fsqrt_rn(x));
    // div: |a|, |b| in [2^-100, 2^100), quotient exponent within +-119
    const int ea = (int)((h >> 40) % 200) - 100;
    int eb = (int)((h2 >> 40) % 200) - 100;
    eb = ea - eb > 119 ? ea - 119 : (eb - ea > 119 ? ea + 119 : eb);
    const float a = __uint_as_float((uint32_t)(h2 >> 63) << 31 | (uint32_t)(ea + 127) << 23 |
                                    ((uint32_t)(h >> 8) & 0x7FFFFFu));
    const float d = __uint_as_float((uint32_t)(eb + 127) << 23 | ((uint32_t)(h2 >> 8) & 0x7FFFFFu));
    bad[2] += __float_as_uint(div_cr(a, d)) != __float_as_uint(__fdiv_rn(a, d));
  }
  for (int k = 0; k < 3; ++k)
    if (bad[k]) atomicAdd(&g_arith_bad[k], (unsigned long long)bad[k]);
}

// Exhaustive check of the certified logarithms' bounds against log1pf / logf:
// every float a in [0, 2^-5] and z in [2^-1, 2^64].  Also records the largest
// errors seen (as double bit patterns, non-negative so unsigned order works):
// [0] max |log1pf - series| / series, [1] max |logf - approx| where |approx| < 1,
// [2] max |logf - approx| / |approx| where |approx| >= 1.
__device__ unsigned long long g_log_bad[2];
__device__ unsigned long long g_log_err[3];

__global__ void __launch_bounds__(kThreads) luma_log_check_kernel() {
  constexpr uint32_t kA0 = 0u, kA1 = 0x3D000000u;           // 0 .. 2^-5
  constexpr uint32_t kZ0 = 0x3F000000u, kZ1 = 0x5F800000u;  // 2^-1 .. 2^64
  constexpr uint64_t kNa = (uint64_t)(kA1 - kA0) + 1, kNz = (uint64_t)(kZ1 - kZ0) + 1;
  unsigned long long bad_m = 0, bad_w = 0;
  double e0 = 0.0, e1 = 0.0, e2 = 0.0;
  for (uint64_t i = (uint64_t)blockIdx.x * kThreads + threadIdx.x; i < kNa + kNz;
       i += (uint64_t)gridDim.x * kThreads) {
    if (i < kNa) {
      const float a = __uint_as_float(kA0 + (uint32_t)i);
      if (!(a <= kCertLog1pMax)) continue;
      const double lc = (double)log1pf(a), la = (double)log1p_series(a);
      const double err = fabs(lc - la);
      if (err > (double)kLog1pRel * la) ++bad_m;
      if (la > 0.0) e0 = fmax(e0, err / la);
    } else {
      const float z = __uint_as_float(kZ0 + (uint32_t)(i - kNa));
      if (!(z >= kCertLogZMin && z <= kCertLogZMax)) continue;
      const double lc = (double)logf(z), la = (double)log_approx(z);
      const double err = fabs(lc - la);
      if (err > (double)kLogAbs + (double)kLogRel * fabs(la)) ++bad_w;
      if (fabs(la) < 1.0) e1 = fmax(e1, err); else e2 = fmax(e2, err / fabs(la));
    }
  }
  if (bad_m) atomicAdd(&g_log_bad[0], bad_m);
  if (bad_w) atomicAdd(&g_log_bad[1], bad_w);
  atomicMax(&g_log_err[0], (unsigned long long)__double_as_longlong(e0));
  atomicMax(&g_log_err[1], (unsigned long long)__double_as_longlong(e1));
  atomicMax(&g_log_err[2], (unsigned long long)__double_as_longlong(e2));
}

// Quantize float32 moments onto a grid (reference optimizer.py:315-321,
// functional.py:133-176): Q_m from m, Q_w from v, uniforms from the Philox
// stream keyed by `seed` (or injected).
__global__ void __launch_bounds__(kThreads) luma_quantize_kernel(
    const float* __restrict__ m, const float* __restrict__ v, int64_t n, const Consts c,
    uint32_t k0, uint32_t k1, uint64_t ctr0, const float* __restrict__ u_m,
    const float* __restrict__ u_w, int16_t* __restrict__ q_m, int16_t* __restrict__ q_w) {
  const int64_t n_pairs = (n + 1) / 2;
  for (int64_t P = (int64_t)blockIdx.x * kThreads + threadIdx.x; P < n_pairs;
       P += (int64_t)gridDim.x * kThreads) {
    float um[2], uw[2];
    if (u_m != nullptr) {
      um[0] = u_m[2 * P] * kUScale; uw[0] = u_w[2 * P] * kUScale;  // exact scaling
      um[1] = (2 * P + 1 < n) ? u_m[2 * P + 1] * kUScale : 0.0f;
      uw[1] = (2 * P + 1 < n) ? u_w[2 * P + 1] * kUScale : 0.0f;
    } else {
      const uint64_t ctr = ctr0 + (uint64_t)P;
      const uint4 r = philox4x32_10(make_uint4((uint32_t)ctr, (uint32_t)(ctr >> 32), 0u, 0u), k0, k1);
      um[0] = u24_scaled(r.x); uw[0] = u24_scaled(r.y); um[1] = u24_scaled(r.z); uw[1] = u24_scaled(r.w);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t e = 2 * P + h;
      if (e < n) {
        q_m[e] = (int16_t)quant_m(c, m[e], um[h]);
        q_w[e] = (int16_t)(uint16_t)quant_w(c, v[e], uw[h]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

struct DeviceInfo {
  bool ready = false;
  int status = LUMA_OK;
  int sms = 0;
  int ctas_pass1 = 0;
  int ctas_pass2 = 0;
  PassAccum* noalloc_acc = nullptr;  // device address of g_noalloc_accum
};

constexpr int kMaxDevices = 64;
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

int device_info(DeviceInfo** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(LUMA_ERR_INVALID, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo& di = g_dev[dev];
  if (!di.ready) {
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
    if (prop.major != 10) {
      return fail(LUMA_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a",
                  dev, prop.major, prop.minor);
    }
    e = cudaFuncSetAttribute(luma_pass_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kPass1SmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(pass1)");
    e = cudaFuncSetAttribute(luma_pass_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kPass2SmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(pass2)");
    e = cudaFuncSetAttribute(luma_pass_kernel<false, true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPass1SmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(pass1 noalloc)");
    e = cudaFuncSetAttribute(luma_pass_kernel<true, true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPass2SmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(pass2 noalloc)");
    int b1 = 0, b2 = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b1, luma_pass_kernel<false>, kThreadsPass1,
                                                      kPass1SmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "occupancy(pass1)");
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b2, luma_pass_kernel<true>, kThreadsPass2,
                                                      kPass2SmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "occupancy(pass2)");
    di.sms = prop.multiProcessorCount;
    di.ctas_pass1 = di.sms * (b1 > 0 ? b1 : 1);
    di.ctas_pass2 = di.sms * (b2 > 0 ? b2 : 1);
    di.ready = true;
  }
  *out = &di;
  return LUMA_OK;
}

// max_ctas from LumaStepArgs: 0 = the device default
int cap(int device_ctas, int32_t max_ctas) {
  return (max_ctas > 0 && max_ctas < device_ctas) ? max_ctas : device_ctas;
}

int grid_for(int64_t total_octets, int threads, int max_ctas) {
  // at least one full tile (one octet per thread) per CTA
  const int64_t want = (total_octets + threads - 1) / threads;
  return (int)(want < max_ctas ? (want > 0 ? want : 1) : max_ctas);
}

// Address of g_noalloc_accum on the current device, fetched once per device
// (with that device current) on the first luma_step_noalloc call there.
int noalloc_scratch(DeviceInfo* di, PassAccum** out) {
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (di->noalloc_acc == nullptr) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_accum);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(noalloc scratch)");
    di->noalloc_acc = static_cast<PassAccum*>(ptr);
  }
  *out = di->noalloc_acc;
  return LUMA_OK;
}

}  // namespace

thread_local char luma_g_err[512] = "";

int luma_fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(luma_g_err, sizeof(luma_g_err), fmt, ap);
  va_end(ap);
  return code;
}

int luma_cuda_fail(cudaError_t e, const char* what) {
  return luma_fail(LUMA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

extern "C" {

int luma_abi_version(void) { return LUMA_ABI_VERSION; }

const char* luma_last_error(void) { return luma_g_err; }

int luma_error_flags(uint32_t* out, int clear) {
  luma_g_err[0] = '\0';
  if (out == nullptr) return fail(LUMA_ERR_INVALID, "luma_error_flags: out is null");
  unsigned int v = 0u;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_kernel_error, sizeof(v));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyFromSymbol(error flags)");
  if (clear && v != 0u) {
    const unsigned int zero = 0u;
    e = cudaMemcpyToSymbol(g_kernel_error, &zero, sizeof(zero));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyToSymbol(error flags)");
  }
  *out = v;
  return LUMA_OK;
}

int luma_launch_config(int32_t* out, int n) {
  const int32_t v[8] = {kThreadsPass1, 8, kP1Stages, kThreadsPass2, 4, kHotStages / 2, 1,
                        (int32_t)kLutMinElems};
  if (out == nullptr || n <= 0) return 0;
  const int k = n < 8 ? n : 8;
  for (int i = 0; i < k; ++i) out[i] = v[i];
  return k;
}

int luma_struct_sizes(int64_t* out, int n) {
  const int64_t sizes[5] = {(int64_t)sizeof(LumaTensorDesc), (int64_t)sizeof(LumaStepRow),
                            (int64_t)sizeof(LumaGrid), (int64_t)sizeof(LumaSlot),
                            (int64_t)sizeof(LumaStepArgs)};
  if (out == nullptr || n <= 0) return 0;
  const int k = n < 5 ? n : 5;
  for (int i = 0; i < k; ++i) out[i] = sizes[i];
  return k;
}

int luma_step(const LumaStepArgs* args, void* stream) {
  luma_g_err[0] = '\0';
  if (args == nullptr) return fail(LUMA_ERR_INVALID, "luma_step: args is NULL");
  const LumaStepArgs a = *args;
  if (a.n_desc < 0 || a.n_rows < 0 || a.total_octets < 0 || a.max_ctas < 0)
    return fail(LUMA_ERR_INVALID,
                "luma_step: negative size (n_desc=%d n_rows=%d total_octets=%lld max_ctas=%d)",
                a.n_desc, a.n_rows, (long long)a.total_octets, a.max_ctas);
  if (a.n_desc == 0 || a.total_octets == 0) return LUMA_OK;
  if (a.descs == nullptr || a.slots == nullptr || a.rows == nullptr || a.n_rows == 0)
    return fail(LUMA_ERR_INVALID, "luma_step: descs/slots/rows must be non-NULL and n_rows > 0");
  DeviceInfo* di = nullptr;
  int st = device_info(&di);
  if (st != LUMA_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (a.events[0]) {
    e = cudaEventRecord(static_cast<cudaEvent_t>(a.events[0]), s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
  }
  luma_pass_kernel<false><<<grid_for(a.total_octets, kThreadsPass1, cap(di->ctas_pass1, a.max_ctas)), kThreadsPass1,
                            kPass1SmemBytes, s>>>(a, 1, nullptr);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch pass 1");
  if (a.events[1]) {
    e = cudaEventRecord(static_cast<cudaEvent_t>(a.events[1]), s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
  }
  luma_pass_kernel<true><<<grid_for(a.total_octets, kThreadsPass2, cap(di->ctas_pass2, a.max_ctas)), kThreadsPass2,
                           kPass2SmemBytes, s>>>(a, 1, nullptr);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch pass 2");
  if (a.step_counters != nullptr) {
    luma_count_steps_kernel<<<(a.n_desc + kThreads - 1) / kThreads, kThreads, 0, s>>>(
        a.descs, a.n_desc, a.step_counters, a.found_inf);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "launch step count");
  }
  if (a.events[2]) {
    e = cudaEventRecord(static_cast<cudaEvent_t>(a.events[2]), s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
  }
  return LUMA_OK;
}

int luma_arith_selfcheck(uint64_t n, uint64_t seed, uint64_t* mismatches, void* stream) {
  luma_g_err[0] = '\0';
  if (mismatches == nullptr) return fail(LUMA_ERR_INVALID, "luma_arith_selfcheck: NULL pointer");
  DeviceInfo* di = nullptr;
  int st = device_info(&di);
  if (st != LUMA_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned long long zero[3] = {0ull, 0ull, 0ull};
  cudaError_t e = cudaMemcpyToSymbolAsync(g_arith_bad, zero, sizeof(zero), 0,
                                          cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyToSymbolAsync(selfcheck)");
  if (n > 0) {
    const uint64_t want = (n + kThreads - 1) / kThreads;
    const int blocks = (int)(want < (uint64_t)di->sms * 8 ? want : (uint64_t)di->sms * 8);
    luma_arith_check_kernel<<<blocks, kThreads, 0, s>>>(n, seed);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "launch arith selfcheck");
  }
  unsigned long long out[3];
  e = cudaMemcpyFromSymbolAsync(out, g_arith_bad, sizeof(out), 0, cudaMemcpyDeviceToHost, s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyFromSymbolAsync(selfcheck)");
  e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize(selfcheck)");
  for (int k = 0; k < 3; ++k) mismatches[k] = out[k];
  return LUMA_OK;
}

int luma_log_selfcheck(uint64_t* violations, double* max_err, void* stream) {
  luma_g_err[0] = '\0';
  if (violations == nullptr || max_err == nullptr)
    return fail(LUMA_ERR_INVALID, "luma_log_selfcheck: NULL pointer");
  DeviceInfo* di = nullptr;
  int st = device_info(&di);
  if (st != LUMA_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned long long zero[3] = {0ull, 0ull, 0ull};
  cudaError_t e = cudaMemcpyToSymbolAsync(g_log_bad, zero, 2 * sizeof(zero[0]), 0,
                                          cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess)
    e = cudaMemcpyToSymbolAsync(g_log_err, zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyToSymbolAsync(log selfcheck)");
  luma_log_check_kernel<<<di->sms * 8, kThreads, 0, s>>>();
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch log selfcheck");
  unsigned long long bad[2], err[3];
  e = cudaMemcpyFromSymbolAsync(bad, g_log_bad, sizeof(bad), 0, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess)
    e = cudaMemcpyFromSymbolAsync(err, g_log_err, sizeof(err), 0, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "log selfcheck readback");
  violations[0] = bad[0];
  violations[1] = bad[1];
  for (int k = 0; k < 3; ++k) memcpy(&max_err[k], &err[k], sizeof(double));
  return LUMA_OK;
}

int luma_decode(const int16_t* q_m, const int16_t* q_w, int64_t numel, float dm, float w_min,
                float dw, float eps32, float* exp_avg, float* exp_avg_sq, void* stream) {
  luma_g_err[0] = '\0';
  if (numel < 0) return fail(LUMA_ERR_INVALID, "luma_decode: negative numel");
  if (numel == 0) return LUMA_OK;
  if (!q_m || !q_w || !exp_avg || !exp_avg_sq)
    return fail(LUMA_ERR_INVALID, "luma_decode: NULL pointer");
  DeviceInfo* di = nullptr;
  int st = device_info(&di);
  if (st != LUMA_OK) return st;
  const int64_t blocks_needed = (numel + kThreads - 1) / kThreads;
  const int blocks = (int)(blocks_needed < di->sms * 8 ? blocks_needed : di->sms * 8);
  luma_decode_kernel<<<blocks, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      q_m, q_w, numel, dm, w_min, dw, eps32, exp_avg, exp_avg_sq);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch decode");
  return LUMA_OK;
}


int luma_quantize(const float* m, const float* v, int64_t numel, const LumaGrid* grid,
                  float eps32, float w_max, int64_t seed, int64_t rng_offset, const float* u_m,
                  const float* u_w, int16_t* q_m, int16_t* q_w, void* stream) {
  luma_g_err[0] = '\0';
  if (numel < 0) return fail(LUMA_ERR_INVALID, "luma_quantize: negative numel");
  if (numel == 0) return LUMA_OK;
  if (!m || !v || !grid || !q_m || !q_w)
    return fail(LUMA_ERR_INVALID, "luma_quantize: NULL pointer");
  if ((u_m == nullptr) != (u_w == nullptr))
    return fail(LUMA_ERR_INVALID, "luma_quantize: u_m and u_w must both be set or both NULL");
  if (rng_offset < 0 || (rng_offset & 1))
    return fail(LUMA_ERR_INVALID, "luma_quantize: rng_offset must be even and >= 0");
  DeviceInfo* di = nullptr;
  int st = device_info(&di);
  if (st != LUMA_OK) return st;
  Consts c;
  memset(&c, 0, sizeof(c));
  const LumaGrid& gr = *grid;
  c.eps32 = eps32; c.w_max = w_max;
  c.n_sm32 = gr.s_m32; c.n_dm = gr.dm; c.n_inv_dm = gr.inv_dm; c.n_inv_zm = gr.inv_zm;
  c.n_wmin = gr.w_min; c.n_inv_wmin = gr.inv_wmin; c.n_dw = gr.dw; c.n_inv_dw = gr.inv_dw;
  c.n_inv_zw = gr.inv_zw; c.n_dw_pos = gr.dw_pos;
  c.margin_m = decision_margin(gr.dm);
  c.margin_w = decision_margin(gr.dw);
  c.inv_zm24 = gr.inv_zm * kUScale;
  c.inv_zw24 = gr.inv_zw * kUScale;
  const uint64_t sd = (uint64_t)seed;
  const int64_t n_pairs = (numel + 1) / 2;
  const int64_t want = (n_pairs + kThreads - 1) / kThreads;
  const int blocks = (int)(want < di->sms * 8 ? want : di->sms * 8);
  luma_quantize_kernel<<<blocks, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      m, v, numel, c, (uint32_t)sd, (uint32_t)(sd >> 32), (uint64_t)rng_offset >> 1, u_m, u_w,
      q_m, q_w);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch quantize");
  return LUMA_OK;
}

int luma_step_noalloc(const LumaStepArgs* args, void* stream) {
  luma_g_err[0] = '\0';
  if (args == nullptr) return fail(LUMA_ERR_INVALID, "luma_step_noalloc: args is NULL");
  const LumaStepArgs a = *args;
  if (a.n_desc < 0 || a.n_rows < 0 || a.total_octets < 0 || a.max_ctas < 0)
    return fail(LUMA_ERR_INVALID,
                "luma_step_noalloc: negative size (n_desc=%d n_rows=%d total_octets=%lld "
                "max_ctas=%d)",
                a.n_desc, a.n_rows, (long long)a.total_octets, a.max_ctas);
  if (a.n_desc > LUMA_NOALLOC_MAX_DESCS)
    return fail(LUMA_ERR_INVALID,
                "luma_step_noalloc: %d tensors exceed the built-in scratch of %d; use luma_step "
                "with caller-provided slots for larger tables",
                a.n_desc, LUMA_NOALLOC_MAX_DESCS);
  if (a.n_desc == 0 || a.total_octets == 0) return LUMA_OK;
  if (a.descs == nullptr || a.slots == nullptr || a.rows == nullptr || a.n_rows == 0)
    return fail(LUMA_ERR_INVALID,
                "luma_step_noalloc: descs/slots/rows must be non-NULL and n_rows > 0");
  DeviceInfo* di = nullptr;
  int st = device_info(&di);
  if (st != LUMA_OK) return st;
  PassAccum* acc = nullptr;
  st = noalloc_scratch(di, &acc);
  if (st != LUMA_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The array keeps the previous call's contents; the accumulators must start
  // at zero (a completed call leaves them zero, an aborted one may not).
  cudaError_t e = cudaMemsetAsync(acc, 0, sizeof(PassAccum) * (size_t)a.n_desc, s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(noalloc scratch)");
  if (a.events[0]) {
    e = cudaEventRecord(static_cast<cudaEvent_t>(a.events[0]), s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
  }
  luma_pass_kernel<false, true><<<grid_for(a.total_octets, kThreadsPass1, cap(di->ctas_pass1, a.max_ctas)),
                                  kThreadsPass1, kPass1SmemBytes, s>>>(a, 1, acc);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch pass 1 (noalloc)");
  if (a.events[1]) {
    e = cudaEventRecord(static_cast<cudaEvent_t>(a.events[1]), s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
  }
  luma_pass_kernel<true, true><<<grid_for(a.total_octets, kThreadsPass2, cap(di->ctas_pass2, a.max_ctas)),
                                 kThreadsPass2, kPass2SmemBytes, s>>>(a, 1, acc);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch pass 2 (noalloc)");
  if (a.step_counters != nullptr) {
    luma_count_steps_kernel<<<(a.n_desc + kThreads - 1) / kThreads, kThreads, 0, s>>>(
        a.descs, a.n_desc, a.step_counters, a.found_inf);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "launch step count");
  }
  if (a.events[2]) {
    e = cudaEventRecord(static_cast<cudaEvent_t>(a.events[2]), s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
  }
  return LUMA_OK;
}

}  // extern "C"
