// Fused PPO minibatch loss and its gradient (the loss of rsl-rl's PPO, as
// duck_gym_b200/ppo.py restates it for a Gaussian policy with a
// state-independent std):
//
//   log p_i  = sum_k -(a_ik - mu_ik)^2 / (2 s_k^2) - log s_k - log sqrt(2 pi)
//   r_i      = exp(log p_i - old log p_i)
//   surr     = mean_i max(-A_i r_i, -A_i clamp(r_i, 1 - eps, 1 + eps))
//   c_i      = V'_i + clamp(v_i - V'_i, -eps, eps)        (V' = rollout values)
//   vloss    = mean_i max((v_i - R_i)^2, (c_i - R_i)^2)
//   entropy  = sum_k 1/2 + log sqrt(2 pi) + log s_k       (the same for every row)
//   loss     = surr + c_v vloss - c_e entropy
//   kl       = mean_i sum_k log(s_k / s'_ik + 1e-5)
//                        + (s'_ik^2 + (mu'_ik - mu_ik)^2) / (2 s_k^2) - 1/2
//
// One pass computes every term and the gradient of the loss with respect to
// mu [B, A], s [A] and v [B], with autograd's conventions for the piecewise
// parts (a tie of max sends half the gradient each way; clamp passes the
// gradient on its closed interval), so it can stand in for the ~80 small
// element-wise kernels of the torch expression and their backward.
//
// Kernels: ppoLossRows -- one thread per row: the row's gradients, and
// per-block partial sums of surr, vloss, kl and of the row terms of
// dloss/ds_k; ppoLossFinish -- one block: fixed-order sums of the partials,
// the four statistics, the loss and dloss/ds.  The result does not depend on
// the launch (no atomics).
#pragma once
#include <cuda_runtime.h>
#include <math.h>

namespace duckb200 {

constexpr int kPpoMaxActions = 32;
constexpr int kPpoThreads = 256;
// Partial sums per block: surr, vloss, kl, then dloss/ds_k for k < A.
__host__ __device__ constexpr int ppoPartials(int actions) { return 3 + actions; }

struct PpoLossArgs {
  int batch, actions;
  const float *mu, *std, *value, *act, *oldLogProb, *oldMu, *oldSigma, *targetValue, *returns, *advantage;
  float clip, valueCoef, entropyCoef;
  float *partials;    // [blocks, 3 + A]
  float *out;         // [5]: surrogate, value loss, entropy, kl, loss
  float *gradMu;      // [B, A]
  float *gradStd;     // [A]
  float *gradValue;   // [B]
};

// d max(a, b) / d a with autograd's tie rule.
__device__ __forceinline__ float maxGradFirst(float a, float b) { return a > b ? 1.f : (a < b ? 0.f : 0.5f); }

// AMAX >= p.actions: loops over actions unroll to AMAX with a guard, so the
// per-action terms stay in registers.
template <int AMAX> __global__ void __launch_bounds__(kPpoThreads) ppoLossRows(PpoLossArgs p) {
  __shared__ float red[kPpoThreads / 32][3 + AMAX];
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int A = p.actions;
  const float invB = 1.f / float(p.batch);
  const float halfLog2Pi = 0.91893853320467274178f;
  float surr = 0.f, vloss = 0.f, kl = 0.f;
  float dstd[AMAX];
#pragma unroll
  for (int k = 0; k < AMAX; ++k) dstd[k] = 0.f;
  if (i < p.batch) {
    // Log-probability of the stored action under the new policy.
    float logp = 0.f;
#pragma unroll
    for (int k = 0; k < AMAX; ++k) {
      if (k >= A) break;
      const float s = p.std[k], d = p.act[i * A + k] - p.mu[i * A + k];
      logp += -(d * d) / (2.f * s * s) - logf(s) - halfLog2Pi;
    }
    const float ratio = expf(logp - p.oldLogProb[i]);
    const float adv = p.advantage[i];
    const float lo = 1.f - p.clip, hi = 1.f + p.clip;
    const float clipped = fminf(fmaxf(ratio, lo), hi);
    const float u = -adv * ratio, w = -adv * clipped;
    surr = fmaxf(u, w);
    // d surr / d ratio: through u, or through the clamp when it passes.
    const float pu = maxGradFirst(u, w), pass = ratio >= lo && ratio <= hi ? 1.f : 0.f;
    const float dr = -adv * (pu + (1.f - pu) * pass);
    const float dlogp = invB * dr * ratio;   // d loss / d log p_i
#pragma unroll
    for (int k = 0; k < AMAX; ++k) {
      if (k >= A) break;
      const float s = p.std[k], d = p.act[i * A + k] - p.mu[i * A + k];
      const float is2 = 1.f / (s * s);
      p.gradMu[i * A + k] = dlogp * d * is2;
      dstd[k] = dlogp * (d * d * is2 / s - 1.f / s);
      const float so = p.oldSigma[i * A + k], dm = p.oldMu[i * A + k] - p.mu[i * A + k];
      kl += logf(s / so + 1e-5f) + (so * so + dm * dm) / (2.f * s * s) - 0.5f;
    }
    // Clipped value loss.
    const float v = p.value[i], tv = p.targetValue[i], R = p.returns[i];
    const float dv = v - tv, cdv = fminf(fmaxf(dv, -p.clip), p.clip);
    const float c = tv + cdv;
    const float a2 = (v - R) * (v - R), b2 = (c - R) * (c - R);
    vloss = fmaxf(a2, b2);
    const float pa = maxGradFirst(a2, b2), cpass = dv >= -p.clip && dv <= p.clip ? 1.f : 0.f;
    p.gradValue[i] = p.valueCoef * invB * (pa * 2.f * (v - R) + (1.f - pa) * 2.f * (c - R) * cpass);
  }
  // Block sums in a fixed order: warp tree, then warp 0 over the warps.
  float vals[3 + AMAX];
  vals[0] = surr; vals[1] = vloss; vals[2] = kl;
#pragma unroll
  for (int k = 0; k < AMAX; ++k) vals[3 + k] = dstd[k];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int q = 0; q < 3 + AMAX; ++q) {
    if (q >= 3 + A) break;
    float x = vals[q];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    if (lane == 0) red[warp][q] = x;
  }
  __syncthreads();
  if (threadIdx.x < 3 + A) {
    float x = 0.f;
    for (int w2 = 0; w2 < kPpoThreads / 32; ++w2) x += red[w2][threadIdx.x];
    p.partials[blockIdx.x * ppoPartials(A) + threadIdx.x] = x;
  }
}

template <int AMAX> __global__ void __launch_bounds__(kPpoThreads) ppoLossFinish(PpoLossArgs p, int blocks) {
  __shared__ float red[kPpoThreads / 32];
  const int A = p.actions, P = ppoPartials(A);
  const float invB = 1.f / float(p.batch);
  const float halfLog2Pi = 0.91893853320467274178f;
  float total[3 + AMAX];
#pragma unroll
  for (int q = 0; q < 3 + AMAX; ++q) {
    if (q >= P) break;
    float x = 0.f;
    for (int b = threadIdx.x; b < blocks; b += blockDim.x) x += p.partials[b * P + q];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = x;
    __syncthreads();
    float sum = 0.f;
    for (int w2 = 0; w2 < kPpoThreads / 32; ++w2) sum += red[w2];
    total[q] = sum;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    float entropy = 0.f;
    for (int k = 0; k < A; ++k) entropy += 0.5f + halfLog2Pi + logf(p.std[k]);
    const float surr = total[0] * invB, vloss = total[1] * invB, kl = total[2] * invB;
    p.out[0] = surr;
    p.out[1] = vloss;
    p.out[2] = entropy;
    p.out[3] = kl;
    p.out[4] = surr + p.valueCoef * vloss - p.entropyCoef * entropy;
#pragma unroll
    for (int k = 0; k < AMAX; ++k)
      if (k < A) p.gradStd[k] = total[3 + k] - p.entropyCoef / p.std[k];
  }
}

}  // namespace duckb200
