// optim.cu - the AdamW step of the AZ-NNUE trainer over a flat fp32
// parameter buffer, in one memory-bound pass (28 bytes per parameter: read
// parameter, moments and gradient, write parameter and moments).
//
// The arithmetic restates candle-nn's AdamW::step (candle-nn 0.10, the
// optimizer of src/az/train_gpu_candle.rs:113-122, :159; decoupled weight
// decay after Loshchilov & Hutter) operation for operation in fp32:
//   m' = (m*b1 + 0) + (g*(1-b1) + 0)
//   v' = (v*b2 + 0) + ((g*g)*(1-b2) + 0)
//   m^ = m'*sm + 0,  v^ = v'*sv + 0       sm = 1/(1-b1^t), sv = 1/(1-b2^t)
//   p' = (p*(1-lr*wd) + 0) - ((m^ / (sqrt(v^)*1 + eps))*lr + 0)
// where each "x*a + c" is one of candle's affine maps (a and c rounded to
// fp32, no fused multiply-add) and the scalar factors are formed in double
// (b^t by repeated squaring, as LLVM's powi runtime does) before rounding.
//
// Two entry points: cnnue_adamw takes the step and hyper-parameters from the
// host; cnnue_adamw_device keeps them in device memory and advances the step
// there, so a CUDA graph that contains it replays correctly step after step.
#include <cstring>

#include "common.cuh"

namespace cnnue {
namespace opt {
namespace {

struct AdamWScalars {
  float b1, omb1, b2, omb2, sm, sv, decay, lr, eps;
};
static_assert(sizeof(AdamWScalars) == sizeof(((cnnue_adamw_state*)nullptr)->scalars), "scalar block");

__device__ __forceinline__ float affine(float x, float a, float c) { return __fadd_rn(__fmul_rn(x, a), c); }

__device__ __forceinline__ void adamw_one(float& p, float& m, float& v, float g, const AdamWScalars& k) {
  const float nm = __fadd_rn(affine(m, k.b1, 0.f), affine(g, k.omb1, 0.f));
  const float nv = __fadd_rn(affine(v, k.b2, 0.f), affine(__fmul_rn(g, g), k.omb2, 0.f));
  const float mh = affine(nm, k.sm, 0.f);
  const float vh = affine(nv, k.sv, 0.f);
  const float den = affine(__fsqrt_rn(vh), 1.f, k.eps);
  const float step = affine(__fdiv_rn(mh, den), k.lr, 0.f);
  p = __fsub_rn(affine(p, k.decay, 0.f), step);
  m = nm;
  v = nv;
}

// The scalars come by value (host form) or from device memory (device form,
// written by adamw_prepare_kernel); `kd` non-null selects the latter.
// grad_scale multiplies every gradient first (one fp32 product: 1 is exact);
// skip (device, optional): nonzero = leave everything as it is.
__global__ void __launch_bounds__(256) adamw_vec4_kernel(float4* __restrict__ p, float4* __restrict__ m,
                                                         float4* __restrict__ v, const float4* __restrict__ g,
                                                         int64_t n4, AdamWScalars k, const AdamWScalars* kd,
                                                         float grad_scale, const float* skip) {
  if (skip && *skip != 0.f) return;
  if (kd) k = *kd;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 pp = p[i], mm = m[i], vv = v[i];
    float4 gg = __ldg(g + i);
    gg = make_float4(__fmul_rn(gg.x, grad_scale), __fmul_rn(gg.y, grad_scale), __fmul_rn(gg.z, grad_scale),
                     __fmul_rn(gg.w, grad_scale));
    adamw_one(pp.x, mm.x, vv.x, gg.x, k);
    adamw_one(pp.y, mm.y, vv.y, gg.y, k);
    adamw_one(pp.z, mm.z, vv.z, gg.z, k);
    adamw_one(pp.w, mm.w, vv.w, gg.w, k);
    p[i] = pp;
    m[i] = mm;
    v[i] = vv;
  }
}

__global__ void adamw_scalar_kernel(float* __restrict__ p, float* __restrict__ m, float* __restrict__ v,
                                    const float* __restrict__ g, int64_t begin, int64_t n, AdamWScalars k,
                                    const AdamWScalars* kd, float grad_scale, const float* skip) {
  if (skip && *skip != 0.f) return;
  if (kd) k = *kd;
  for (int64_t i = begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    adamw_one(p[i], m[i], v[i], __fmul_rn(g[i], grad_scale), k);
}

// b^e for e >= 0 by repeated squaring (the powi runtime routine).
__host__ __device__ double powi(double b, int64_t e) {
  double r = 1.0;
  while (true) {
    if (e & 1) r *= b;
    e /= 2;
    if (e == 0) break;
    b *= b;
  }
  return r;
}

// The scalar factors in double, rounded once to fp32.  Every double
// operation is spelled out (no contraction), so host and device forms agree.
__host__ __device__ AdamWScalars make_scalars(double lr, double beta1, double beta2, double eps, double wd,
                                              int64_t step) {
#ifdef __CUDA_ARCH__
#define DSUB(a, b) __dsub_rn(a, b)
#define DMUL(a, b) __dmul_rn(a, b)
#define DDIV(a, b) __ddiv_rn(a, b)
#else
#define DSUB(a, b) ((a) - (b))
#define DMUL(a, b) ((a) * (b))
#define DDIV(a, b) ((a) / (b))
#endif
  AdamWScalars k;
  k.b1 = (float)beta1;
  k.omb1 = (float)DSUB(1.0, beta1);
  k.b2 = (float)beta2;
  k.omb2 = (float)DSUB(1.0, beta2);
  k.sm = (float)DDIV(1.0, DSUB(1.0, powi(beta1, step)));
  k.sv = (float)DDIV(1.0, DSUB(1.0, powi(beta2, step)));
  k.decay = (float)DSUB(1.0, DMUL(lr, wd));
  k.lr = (float)lr;
  k.eps = (float)eps;
#undef DSUB
#undef DMUL
#undef DDIV
  return k;
}

// Device form: advances the step counter and forms this step's scalars;
// with skip flags (any nonzero) it marks the step skipped (pad[0] = 1) and
// leaves the counter.
__global__ void adamw_prepare_kernel(cnnue_adamw_state* st, const float* skip, int n_skip) {
  bool sk = false;
  for (int i = 0; i < n_skip; ++i) sk |= skip[i] != 0.f;
  st->pad[0] = sk ? 1.f : 0.f;
  if (sk) return;
  st->step += 1;
  const AdamWScalars k = make_scalars(st->lr, st->beta1, st->beta2, st->eps, st->weight_decay, st->step);
  memcpy(st->scalars, &k, sizeof(k));
}

int launch_adamw(float* d_params, float* d_m, float* d_v, const float* d_grads, int64_t n, const AdamWScalars& k,
                 const AdamWScalars* kd, cudaStream_t s, float grad_scale = 1.f, const float* skip = nullptr) {
  const bool aligned = ((uintptr_t)d_params | (uintptr_t)d_m | (uintptr_t)d_v | (uintptr_t)d_grads) % 16 == 0;
  int64_t done = 0;
  if (aligned && n >= 4) {
    const int64_t n4 = n / 4;
    const unsigned blocks = (unsigned)std::min<int64_t>((n4 + 255) / 256, 148 * 8);
    adamw_vec4_kernel<<<blocks, 256, 0, s>>>((float4*)d_params, (float4*)d_m, (float4*)d_v, (const float4*)d_grads,
                                            n4, k, kd, grad_scale, skip);
    if (int st = check_launch_error("adamw_vec4_kernel")) return st;
    done = n4 * 4;
  }
  if (done < n) {
    const unsigned blocks = (unsigned)std::min<int64_t>((n - done + 255) / 256, 148 * 8);
    adamw_scalar_kernel<<<blocks, 256, 0, s>>>(d_params, d_m, d_v, d_grads, done, n, k, kd, grad_scale, skip);
    if (int st = check_launch_error("adamw_scalar_kernel")) return st;
  }
  return CNNUE_OK;
}

// AdamW over up to kMaxRanges disjoint ranges of a flat buffer in one launch
// (device-state scalars, scale 1): the ranges' float4 groups are one index
// space; ranges start and end on 4-element boundaries.
__global__ void __launch_bounds__(256) adamw_ranges_kernel(float* __restrict__ p, float* __restrict__ m,
                                                           float* __restrict__ v, const float* __restrict__ g,
                                                           AdamWRanges r, const AdamWScalars* kd) {
  const AdamWScalars k = *kd;
  int64_t total = 0;
  for (int j = 0; j < r.n; ++j) total += r.len4[j];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t q = i;
    int j = 0;
    while (j + 1 < r.n && q >= r.len4[j]) q -= r.len4[j++];
    const int64_t e = r.begin[j] + 4 * q;
    float4 pp = *(float4*)(p + e), mm = *(float4*)(m + e), vv = *(float4*)(v + e);
    const float4 gg = __ldg((const float4*)(g + e));
    adamw_one(pp.x, mm.x, vv.x, gg.x, k);
    adamw_one(pp.y, mm.y, vv.y, gg.y, k);
    adamw_one(pp.z, mm.z, vv.z, gg.z, k);
    adamw_one(pp.w, mm.w, vv.w, gg.w, k);
    *(float4*)(p + e) = pp;
    *(float4*)(m + e) = mm;
    *(float4*)(v + e) = vv;
  }
}

}  // namespace
}  // namespace opt

int adamw_prepare(cnnue_adamw_state* d_state, cudaStream_t s) {
  opt::adamw_prepare_kernel<<<1, 1, 0, s>>>(d_state, nullptr, 0);
  return check_launch_error("adamw_prepare_kernel");
}

int adamw_ranges(float* d_params, float* d_m, float* d_v, const float* d_grads, const AdamWRanges& r,
                 const cnnue_adamw_state* d_state, cudaStream_t s) {
  int64_t total = 0;
  for (int j = 0; j < r.n; ++j) {
    if ((r.begin[j] & 3) || r.len4[j] < 0) return set_error(CNNUE_ERR_INVALID_ARG, "adamw range not aligned");
    total += r.len4[j];
  }
  if (total == 0) return CNNUE_OK;
  if (((uintptr_t)d_params | (uintptr_t)d_m | (uintptr_t)d_v | (uintptr_t)d_grads) & 15)
    return set_error(CNNUE_ERR_INVALID_ARG, "adamw buffers not 16-byte aligned");
  const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, 148 * 8);
  opt::adamw_ranges_kernel<<<blocks, 256, 0, s>>>(d_params, d_m, d_v, d_grads, r,
                                                   (const opt::AdamWScalars*)d_state->scalars);
  return check_launch_error("adamw_ranges_kernel");
}

}  // namespace cnnue

using namespace cnnue;
using namespace cnnue::opt;

extern "C" {

int cnnue_adamw(float* d_params, float* d_m, float* d_v, const float* d_grads, int64_t n, double lr, double beta1,
                double beta2, double eps, double weight_decay, int64_t step, void* stream) {
  if (n < 0 || (n > 0 && (!d_params || !d_m || !d_v || !d_grads)))
    return set_error(CNNUE_ERR_INVALID_ARG, "null buffer or negative size");
  if (step < 1) return set_error(CNNUE_ERR_INVALID_ARG, "step must be >= 1");
  if (n == 0) return CNNUE_OK;
  return launch_adamw(d_params, d_m, d_v, d_grads, n, make_scalars(lr, beta1, beta2, eps, weight_decay, step),
                      nullptr, (cudaStream_t)stream);
}

int cnnue_adamw_device(float* d_params, float* d_m, float* d_v, const float* d_grads, int64_t n,
                       cnnue_adamw_state* d_state, void* stream) {
  if (n < 0 || !d_state || (n > 0 && (!d_params || !d_m || !d_v || !d_grads)))
    return set_error(CNNUE_ERR_INVALID_ARG, "null buffer or negative size");
  cudaStream_t s = (cudaStream_t)stream;
  adamw_prepare_kernel<<<1, 1, 0, s>>>(d_state, nullptr, 0);
  if (int st = check_launch_error("adamw_prepare_kernel")) return st;
  if (n == 0) return CNNUE_OK;
  return launch_adamw(d_params, d_m, d_v, d_grads, n, AdamWScalars{}, (const AdamWScalars*)d_state->scalars, s);
}

int cnnue_adamw_device_scaled(float* d_params, float* d_m, float* d_v, const float* d_grads, int64_t n,
                              cnnue_adamw_state* d_state, float grad_scale, const float* d_skip, int n_skip,
                              void* stream) {
  if (n < 0 || !d_state || n_skip < 0 || (n_skip > 0 && !d_skip) ||
      (n > 0 && (!d_params || !d_m || !d_v || !d_grads)))
    return set_error(CNNUE_ERR_INVALID_ARG, "null buffer or negative size");
  cudaStream_t s = (cudaStream_t)stream;
  adamw_prepare_kernel<<<1, 1, 0, s>>>(d_state, d_skip, n_skip);
  if (int st = check_launch_error("adamw_prepare_kernel")) return st;
  if (n == 0) return CNNUE_OK;
  return launch_adamw(d_params, d_m, d_v, d_grads, n, AdamWScalars{}, (const AdamWScalars*)d_state->scalars, s,
                      grad_scale, d_state->pad);
}

}  // extern "C"
