// Generalised advantage estimation over a device rollout buffer
// (train/ppo.py:101-110): one thread per env walks t = T-1 .. 0.
//   delta = rew + (gamma * next_val) * nonterm - val
//   gae   = delta + ((gamma*lam) * nonterm) * gae
// with gamma*lam formed in double and rounded once, as the reference's
// Python-scalar products are.

#include "qqt_common.cuh"

namespace qqt {

__global__ void k_gae(const float* __restrict__ rew, int rew_stride, const uint8_t* __restrict__ done,
                      const float* __restrict__ val, int val_stride,
                      const float* __restrict__ last_val, int T, int N, float gamma, float gl,
                      float* __restrict__ adv, float* __restrict__ ret) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= N) return;
  float gae = 0.f;
  float next_val = last_val[e];
  for (int t = T - 1; t >= 0; --t) {
    const float v = val[(size_t)t * val_stride + e];
    const float nonterm = __fsub_rn(1.f, done[(size_t)t * N + e] ? 1.f : 0.f);
    const float delta = __fsub_rn(
        __fadd_rn(rew[(size_t)t * rew_stride + e], __fmul_rn(__fmul_rn(gamma, next_val), nonterm)), v);
    gae = __fadd_rn(delta, __fmul_rn(__fmul_rn(gl, nonterm), gae));
    adv[(size_t)t * N + e] = gae;
    ret[(size_t)t * N + e] = __fadd_rn(gae, v);
    next_val = v;
  }
}

}  // namespace qqt

using namespace qqt;

extern "C" int qqt_gae(const float* rew, int32_t rew_stride, const uint8_t* done, const float* val,
                       int32_t val_stride, const float* last_val, int32_t T, int32_t N,
                       double gamma, double lam, float* adv, float* ret, qqt_stream_t stream) {
  if (!rew || !done || !val || !last_val || !adv || !ret || T <= 0 || N <= 0 || rew_stride < N ||
      val_stride < N)
    return QQT_E_ARG;
  k_gae<<<(N + 255) / 256, 256, 0, (cudaStream_t)stream>>>(rew, rew_stride, done, val, val_stride,
                                                            last_val, T, N, (float)gamma,
                                                            (float)(gamma * lam), adv, ret);
  return launch_status();
}
