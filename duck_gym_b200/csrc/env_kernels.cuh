// Fused tensor-environment kernels: the per-control-step math of the
// reference's TensorEnv (python/duck_gym/tensor_env.py) in one thread per
// environment, reading the physics state straight from the batch's records.
//
//   envTargetsKernel    actions -> clamped action and PD target    (:280-283)
//   envPostStepKernel   frames, termination, reward, time-outs,
//                       episode bookkeeping, terminal observation  (:221-361)
//   envObserveKernel    observation only (get_observations)        (:238-261)
//   envResetBuffers     masked reset of the env buffers            (:196-219)
//
// The reference evaluates this math as ~60 separate torch kernels per step.
// Quantities that decide the termination mask (projected gravity, base
// height, diagnostics, finiteness) are computed with the rounding of the
// reference's CPU torch ops -- each product rounded, 3-term sums left to
// right, cross products as fma(a_i, b_j, -(a_j b_i)) -- so the masks agree bit
// for bit; observations and rewards are within float tolerance.
#pragma once
#include "aux_kernels.cuh"

namespace duckb200 {

struct EnvKernelParams {
  int task, filter, maxEpisode, obsDim, nj;
  // Python scalars of the env: torch casts them to the tensor dtype per op.
  double rootHeight, controlDt, velocityAlpha, trackingWeight, headingWeight, sigma2, phaseRate;
  float tilt;  // -cos(0.5) as a float32 tensor
  double iquat[4];
  // Gait shaping (tensor_env.py:152-171, 263-277, 318-344).
  int gait, footClearance, loadTransfer, gaitSamples, footPoints;
  int footBody[2];
  double gaitPeriod, gaitLift, massG;
  const void *gaitTable;    // [4, samples, J] Real
  const void *footXyz;      // [2, P, 3] Real
};

// Torch CPU cross product: fma(a_i, b_j, -(a_j b_i)).
template <class R> __device__ __forceinline__ V3<R> tcross(V3<R> a, V3<R> b);
template <> __device__ __forceinline__ V3<float> tcross(V3<float> a, V3<float> b) {
  return {__fmaf_rn(a.y, b.z, -__fmul_rn(a.z, b.y)), __fmaf_rn(a.z, b.x, -__fmul_rn(a.x, b.z)),
          __fmaf_rn(a.x, b.y, -__fmul_rn(a.y, b.x))};
}
template <> __device__ __forceinline__ V3<double> tcross(V3<double> a, V3<double> b) {
  return {__fma_rn(a.y, b.z, -__dmul_rn(a.z, b.y)), __fma_rn(a.z, b.x, -__dmul_rn(a.x, b.z)),
          __fma_rn(a.x, b.y, -__dmul_rn(a.y, b.x))};
}
// tensor_env.py:9-18 multiply(a, b).
template <class R> __device__ __forceinline__ Q4<R> tmultiply(Q4<R> a, Q4<R> b) {
  V3<R> av{a.x, a.y, a.z}, bv{b.x, b.y, b.z};
  R s = xadd(xadd(xmul(av.x, bv.x), xmul(av.y, bv.y)), xmul(av.z, bv.z));
  R w = xsub(xmul(a.w, b.w), s);
  V3<R> c = tcross(av, bv);
  return {w, xadd(xadd(xmul(a.w, bv.x), xmul(b.w, av.x)), c.x), xadd(xadd(xmul(a.w, bv.y), xmul(b.w, av.y)), c.y),
          xadd(xadd(xmul(a.w, bv.z), xmul(b.w, av.z)), c.z)};
}
// tensor_env.py:21-23 inverse_rotate(q, v).
template <class R> __device__ __forceinline__ V3<R> tinverseRotate(Q4<R> q, V3<R> v) {
  V3<R> u{-q.x, -q.y, -q.z};
  V3<R> t = tcross(u, v);
  t = {xmul(R(2), t.x), xmul(R(2), t.y), xmul(R(2), t.z)};
  V3<R> c = tcross(u, t);
  return {xadd(xadd(v.x, xmul(q.w, t.x)), c.x), xadd(xadd(v.y, xmul(q.w, t.y)), c.y),
          xadd(xadd(v.z, xmul(q.w, t.z)), c.z)};
}

template <class R> struct EnvFrame {
  V3<R> g, v, w;
  R yaw0, yaw1, height;
  bool finite;
};

template <class R>
__device__ __forceinline__ EnvFrame<R> envFrame(const DevModel<R> *m, const R *rec, const EnvKernelParams &p) {
  const R *bodies = rec + kRecHeader;
  const R *b1 = bodies + kRecBody;
  Q4<R> iq{R(p.iquat[0]), R(p.iquat[1]), R(p.iquat[2]), R(p.iquat[3])};
  Q4<R> q = tmultiply(Q4<R>{b1[3], b1[4], b1[5], b1[6]}, iq);
  EnvFrame<R> f;
  f.g = tinverseRotate(q, V3<R>{R(0), R(0), R(-1)});
  f.v = tinverseRotate(q, V3<R>{b1[7], b1[8], b1[9]});
  f.w = tinverseRotate(q, V3<R>{b1[10], b1[11], b1[12]});
  f.yaw0 = R(1) - R(2) * (q.y * q.y + q.z * q.z);
  f.yaw1 = R(2) * (q.w * q.z + q.x * q.y);
  f.height = xsub(b1[2], R(p.rootHeight));
  bool finite = true;
  for (int b = 0; b < m->nb; ++b)
    for (int k = 0; k < 13; ++k) finite &= isfinite(bodies[kRecBody * b + k]);
  f.finite = finite;
  return f;
}

template <class R>
__device__ __forceinline__ void envWriteObs(const DevModel<R> *m, const R *rec, const EnvKernelParams &p,
                                            const EnvFrame<R> &f, const R *home, const R *actions, long long len,
                                            const R *commands, const R *filtered, float *obs) {
  const R *bodies = rec + kRecHeader;
  int o = 0;
  obs[o++] = float(f.g.x); obs[o++] = float(f.g.y); obs[o++] = float(f.g.z);
  obs[o++] = float(f.v.x); obs[o++] = float(f.v.y); obs[o++] = float(f.v.z);
  obs[o++] = float(f.w.x); obs[o++] = float(f.w.y); obs[o++] = float(f.w.z);
  obs[o++] = float(f.height);
  const int nj = m->nj;
  for (int j = 0; j < nj; ++j) {
    R angle, rate;
    jointState(m, bodies, j, &angle, &rate);
    obs[o + j] = float(angle - home[j]);
    obs[o + nj + j] = float(R(0.1) * rate);
    obs[o + 2 * nj + j] = float(actions[j]);
  }
  o += 3 * nj;
  if (p.task == 1) {
    obs[o++] = float(commands[0]);
    obs[o++] = float(commands[1]);
    obs[o++] = float(f.yaw0);
    obs[o++] = float(f.yaw1);
    R phase = R(len) * R(p.controlDt) * R(p.phaseRate);   // phaseRate = 2 pi / gait period
    obs[o++] = float(sin(phase));
    obs[o++] = float(cos(phase));
  }
  if (p.filter) {
    obs[o++] = float(filtered[0]);
    obs[o++] = float(filtered[1]);
  }
}

// a = clamp(actions, -1, 1); target = clamp(home + scale a, lower, upper).
template <class R>
__global__ void envTargetsKernel(int count, int nj, const R *actions, R scale, const R *home, const R *lower,
                                 const R *upper, R *aOut, R *targetOut) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= count * nj) return;
  const int j = i % nj;
  R a = rclamp(actions[i], R(-1), R(1));
  aOut[i] = a;
  targetOut[i] = rmin(rmax(xadd(home[j], xmul(scale, a)), lower[j]), upper[j]);
}

// tensor_env.py:263-283 with the gait table: reference target of each env
// (the table at the episode phase, in the direction the command points to,
// blended in over the first second), then the clamped PD target.  One thread
// per (env, joint).
template <class R>
__global__ void envGaitTargetsKernel(int count, EnvKernelParams p, const R *actions, R scale, const R *home,
                                     const R *lower, const R *upper, const long long *episodeLength,
                                     const R *commands, R *aOut, R *targetOut) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int nj = p.nj;
  if (i >= count * nj) return;
  const int e = i / nj, j = i % nj;
  const R len = R(episodeLength[e]);
  R ref = home[j];
  if (p.gait) {
    const R phase = len * R(p.controlDt) / R(p.gaitPeriod);
    const int n = p.gaitSamples;
    const R index = (phase - floor(phase)) * R(n);
    const int lo = int(index);
    const R fraction = index - R(lo);
    const R cx = commands[2 * size_t(e)], cy = commands[2 * size_t(e) + 1];
    // argmax over the directions (+x, -x, +y, -y), first one on ties.
    const R dots[4] = {cx, -cx, cy, -cy};
    int d = 0;
    for (int k = 1; k < 4; ++k)
      if (dots[k] > dots[d]) d = k;
    const R *table = static_cast<const R *>(p.gaitTable) + size_t(d) * n * nj;
    const R r = table[size_t(lo) * nj + j] * (R(1) - fraction) + table[size_t((lo + 1) % n) * nj + j] * fraction;
    const R blend = rmin(rmax(len * R(p.controlDt), R(0)), R(1));
    ref = home[j] + (r - home[j]) * blend;
  }
  const R a = rclamp(actions[i], R(-1), R(1));
  aOut[i] = a;
  targetOut[i] = rmin(rmax(xadd(ref, xmul(scale, a)), lower[j]), upper[j]);
}

// Foot-clearance and load-transfer shaping (tensor_env.py:318-344), added to
// the reward before the failure override.
template <class R>
__device__ __forceinline__ R gaitShaping(const DevModel<R> *m, const R *rec, const EnvKernelParams &p, long long len) {
  const R *bodies = rec + kRecHeader;
  R penalty = R(0);
  if (p.footClearance) {
    const R *pts = static_cast<const R *>(p.footXyz);
    R sum = R(0);
    for (int f = 0; f < 2; ++f) {
      const R *fb = bodies + kRecBody * p.footBody[f];
      const V3<R> up = tinverseRotate(Q4<R>{fb[3], fb[4], fb[5], fb[6]}, V3<R>{R(0), R(0), R(1)});
      R lowest = R(INFINITY);
      for (int v = 0; v < p.footPoints; ++v) {
        const R *q = pts + (size_t(f) * p.footPoints + v) * 3;
        lowest = rmin(lowest, q[0] * up.x + q[1] * up.y + q[2] * up.z + fb[2]);
      }
      R phase = (R(len) + R(1)) * R(p.controlDt) / R(p.gaitPeriod) + (f ? R(0.5) : R(0));
      phase = phase - floor(phase);
      const R swing = rmin(rmax((phase - R(0.6)) / R(0.4), R(0)), R(1));
      const R s = sin(R(3.14159265358979323846) * swing);
      const R desired = R(p.gaitLift) * (s * s);
      const R err = rmax(lowest, R(0)) - desired;
      sum += err * err;
    }
    penalty += R(20000) * sum;
  }
  if (p.loadTransfer) {
    const R cycle = (R(len) + R(1)) * R(p.controlDt) / R(p.gaitPeriod);
    const R left = R(0.5) + R(0.5) * sin(R(2 * 3.14159265358979323846) * (cycle - R(0.05)));
    const R wanted[2] = {left, R(1) - left};
    R sum = R(0);
    for (int f = 0; f < 2; ++f) {
      const R fz = envBodyForce(m, rec, p.footBody[f]).z / R(p.massG);
      const R err = rmin(rmax(fz, R(0)), R(3)) - wanted[f];
      sum += err * err;
    }
    penalty += R(3) * sum;
  }
  return penalty;
}

template <class R>
__global__ void envPostStepKernel(const DevModel<R> *__restrict__ m, const R *records, int stride, int count,
                                  EnvKernelParams p, const R *home, const R *actions, R *prevActions,
                                  long long *episodeLength, float *returns, const R *commands, R *filtered,
                                  float *obs, float *reward, bool *failedOut, bool *timeoutOut, bool *doneOut,
                                  R *diagOut, float *tracking) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= count) return;
  const int nj = m->nj;
  const R *rec = records + size_t(e) * stride;
  const R *bodies = rec + kRecHeader;
  const EnvFrame<R> f = envFrame(m, rec, p);
  const bool failed = f.g.z > R(p.tilt) || fabs(f.height) > R(0.04) || rec[2] > R(0.005) || rec[3] > R(0.005) ||
                      rec[0] > R(0) || !f.finite;
  const R *a = actions + size_t(e) * nj;
  R *prev = prevActions + size_t(e) * nj;
  R sa = R(0), sd = R(0), sj = R(0);
  for (int j = 0; j < nj; ++j) {
    R angle, rate;
    jointState(m, bodies, j, &angle, &rate);
    R dj = angle - home[j], da = a[j] - prev[j];
    sj += dj * dj;
    sa += a[j] * a[j];
    sd += da * da;
  }
  const R g2 = f.g.x * f.g.x + f.g.y * f.g.y, h2 = f.height * f.height;
  const R ww = dot(f.w, f.w);
  R r;
  R *filt = filtered + 2 * size_t(e);
  const R *cmd = commands + 2 * size_t(e);
  if (diagOut) {
    R *o = diagOut + 6 * size_t(e);
    o[0] = rec[2]; o[1] = rec[3]; o[2] = rec[4]; o[3] = rec[5]; o[4] = rec[6]; o[5] = rec[0];
  }
  if (p.task == 1) {
    const R *b1 = bodies + kRecBody;
    R vx = b1[7], vy = b1[8];
    const R ix = vx - cmd[0], iy = vy - cmd[1];
    if (p.filter) {
      const R alpha = R(p.velocityAlpha);
      filt[0] = (R(1) - alpha) * filt[0] + alpha * vx;
      filt[1] = (R(1) - alpha) * filt[1] + alpha * vy;
      vx = filt[0];
      vy = filt[1];
    }
    const R ex = vx - cmd[0], ey = vy - cmd[1];
    const R error = ex * ex + ey * ey;
    if (tracking) {
      // Per-env terms of the reference's tracking/* log entries (tensor_env.py:377-387).
      float *t = tracking + 4 * size_t(e);
      t[0] = float(sqrt(ix * ix + iy * iy));
      t[1] = float(b1[7] * cmd[0] + b1[8] * cmd[1]);
      t[2] = float(sqrt(error));
      t[3] = float(fabs(atan2(f.yaw1, f.yaw0)));
    }
    r = exp(R(-20) * g2) + exp(R(-2000) * h2) + R(p.trackingWeight) * exp(-error / R(p.sigma2)) -
        R(0.1) * ww - R(p.headingWeight) * (R(1) - f.yaw0) - R(0.02) * sa - R(0.03) * sd;
  } else {
    r = R(1.5) * exp(R(-20) * g2) + exp(R(-2000) * h2) + R(0.5) * exp(R(-10) * dot(f.v, f.v)) - R(0.02) * ww -
        R(0.05) * sj - R(0.01) * sa - R(0.02) * sd;
  }
  if (p.footClearance || p.loadTransfer) r -= gaitShaping(m, rec, p, episodeLength[e]);
  r = (failed ? R(-2) : r) * R(p.controlDt);
  const long long len = episodeLength[e] + 1;
  episodeLength[e] = len;
  returns[e] += float(r);
  reward[e] = float(r);
  for (int j = 0; j < nj; ++j) prev[j] = a[j];
  const bool timeout = len >= p.maxEpisode && !failed;
  failedOut[e] = failed;
  timeoutOut[e] = timeout;
  doneOut[e] = failed || timeout;
  envWriteObs(m, rec, p, f, home, a, len, cmd, filt, obs + size_t(e) * p.obsDim);
}

template <class R>
__global__ void envObserveKernel(const DevModel<R> *__restrict__ m, const R *records, int stride, int count,
                                 EnvKernelParams p, const R *home, const R *actions, const long long *episodeLength,
                                 const R *commands, const R *filtered, float *obs) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= count) return;
  const R *rec = records + size_t(e) * stride;
  const EnvFrame<R> f = envFrame(m, rec, p);
  envWriteObs(m, rec, p, f, home, actions + size_t(e) * m->nj, episodeLength[e], commands + 2 * size_t(e),
              filtered + 2 * size_t(e), obs + size_t(e) * p.obsDim);
}

// tensor_env.py:197-219: zero the buffers of the reset environments and give
// them their new commands.
template <class R>
__global__ void envResetBuffersKernel(int count, int nj, const bool *mask, R *prevActions, R *forces,
                                      long long *episodeLength, float *returns, R *filtered, R *commands,
                                      const R *newCommands) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= count || !mask[e]) return;
  for (int j = 0; j < nj; ++j) prevActions[size_t(e) * nj + j] = R(0);
  for (int k = 0; k < 3; ++k) forces[3 * size_t(e) + k] = R(0);
  episodeLength[e] = 0;
  returns[e] = 0.f;
  filtered[2 * size_t(e)] = filtered[2 * size_t(e) + 1] = R(0);
  if (newCommands) {
    commands[2 * size_t(e)] = newCommands[2 * size_t(e)];
    commands[2 * size_t(e) + 1] = newCommands[2 * size_t(e) + 1];
  }
}

}  // namespace duckb200
