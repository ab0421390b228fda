// Fused kernels of the BAM environment (the reference's
// python/duck_gym/bam_env.py with actuator.py and walking_reward.py), one
// thread per environment, reading the physics state straight from the batch's
// records:
//
//   bamBeginKernel      step prologue: action history, observed velocity,
//                       self-contact maxima cleared, step counter  (:292-303)
//   bamLoadsKernel      RNEA generalized loads (shared-memory arrays) and
//                       the servo's supply voltage                (:305-314)
//   bamServoJointKernel delay ring and the XL330/m6 servo, one thread per
//                       (env, joint) -> motor channels            (:305-331)
//   (physics: advanceMotor of duck_b200.cu, one substep)
//   bamAfterKernel      foot contacts, air / contact timers, self-contact
//                       maxima, mean-velocity filter, ring cursor (:332-344)
//   bamControlKernel    frames, walking reward, failure, time-outs, heading
//                       command, actor / critic observations      (:136-211,
//                       345-418; walking_reward.py:45-122)
//   bamResetKernel      masked reset of the env buffers           (:245-275)
//
// The reference evaluates this as ~40 torch ops per substep plus ~150 per
// control step.  Quantities that decide the failure mask (projected gravity,
// diagnostics, self penetration, finiteness) are computed with the rounding of
// the reference's CPU torch ops, so the masks agree bit for bit; the rest is
// within float tolerance.
#pragma once
#include "env_kernels.cuh"

namespace duckb200 {

enum { kBamTerms = 19 };
// Terms in the reference's order (walking_reward.py:75-96, then the optional
// ones bam_env.py:358-381).
enum {
  tTrackLin, tTrackAng, tUpright, tPose, tBodyAngVel, tAngMomentum, tDofLimits, tActionRate, tAirTime,
  tFootClearance, tFootSwing, tFootSlip, tSelfCollisions, tHeadTracking, tHeadBias, tHeadPosition, tHeadVelocity,
  tTrackMeanVelocity, tTrackHeading
};
// Feature row: root quaternion, gravity, body angular and linear velocity,
// root-origin world velocity, sole-site positions and velocities.
// The last slot holds the sticky numeric-failure flag (diag[:, 5]).
enum { fQuat = 0, fGravity = 4, fAngVel = 7, fLinVel = 10, fOrigin = 13, fSitePos = 16, fSiteVel = 22, fFailed = 28, kFeatures = 29 };

struct BamKernelParams {
  int nj, lag, maxEpisode, sourceIteration, neutralHead, headingHold, reward;
  int headMask, extras, overrideMask, criticDim;
  int footBody[2];
  double dt, stepDt, kpFw, vin, vinDrop, vinMin, forceLimit;
  double kt, res, fBase, fStribeck, lfe, lfm, lfes, lfms, lfeq, lfmq, dthetaStribeck, alpha, fViscous;
  double iquat[4], site[2][3];
  double linVar, vertVar, meanAlpha, meanVar, meanWeight, headingWeight, headingVar, headPosWeight, headVelWeight;
  double tiltLimit;
  double overrides[15];
  double stand[kMaxJoints], walk[kMaxJoints], soft[kMaxJoints][2];
};
enum { xHeadStability = 1, xMeanVelocity = 2, xHeading = 4 };

template <class R> struct BamBuffers {
  const R *home, *rootOffset;
  R *action, *oldAction, *prevMotor, *prevApplied, *observedVelocity, *command, *meanVelocity, *targetYaw;
  R *airTime, *contactTime, *contactForce, *selfContacts, *selfPenetration, *joints, *headEma, *peakHeight;
  R *history, *motor, *features, *terms, *servoSupply;
  bool *contact, *histInit, *done, *timeout, *failed;
  long long *episodeLength;
  int *counters;  // [0] delay-ring cursor, [1] common step counter
  float *obsActor, *obsCritic, *reward;
  const R *envMass = nullptr, *envInertia = nullptr;  // the batch's randomised parameters, if any
};

// torch.lerp on the CPU: start + w (end - start) below w = 0.5, else
// end - (end - start)(1 - w).
template <class R> __device__ __forceinline__ R tlerp(R start, R end, R w) {
  return w < R(0.5) ? start + w * (end - start) : end - (end - start) * (R(1) - w);
}

template <class R> __device__ __forceinline__ V3<R> recV3(const R *p) { return V3<R>{p[0], p[1], p[2]}; }

// ---------------------------------------------------------------- prologue
template <class R>
__global__ void bamBeginKernel(BamKernelParams p, BamBuffers<R> B, int count, const R *actions) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= count) return;
  const int nj = p.nj;
  for (int j = 0; j < nj; ++j) {
    const size_t i = size_t(e) * nj + j;
    B.oldAction[i] = B.action[i];
    B.action[i] = (p.neutralHead && (p.headMask >> j & 1)) ? R(0) : actions[i];
    B.observedVelocity[i] = B.joints[2 * i + 1];
  }
  B.selfContacts[e] = R(0);
  B.selfPenetration[e] = R(0);
  if (e == 0) B.counters[1] += 1;
}

// ---------------------------------------------------------------- servo
// actuator.py:16-77 in two kernels.  bamLoadsKernel: one thread per
// environment, 32 per block, RNEA loads with their per-body arrays in shared
// memory; the hinge loads go to the motor-channel buffer (scratch until the
// joint kernel overwrites it) and the supply voltage to servoSupply.
// bamServoJointKernel: one thread per (environment, joint): delay ring and
// the servo equations, writing the motor channels and the servo history.
template <class R>
__global__ void bamLoadsKernel(const DevModel<R> *__restrict__ m, const R *records, int stride, int count,
                               BamKernelParams p, BamBuffers<R> B) {
  extern __shared__ __align__(16) unsigned char rneaRaw[];
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= count) return;
  const int nj = p.nj;
  RneaShared<R> st{reinterpret_cast<R *>(rneaRaw), m->nb, int(blockDim.x), int(threadIdx.x)};
  const R *off = B.rootOffset + 3 * size_t(e);
  rneaLoads(m, records + size_t(e) * stride, V3<R>{off[0], off[1], off[2]}, B.motor + size_t(e) * nj * 3,
            B.envMass ? B.envMass + size_t(e) * m->nb : nullptr,
            B.envInertia ? B.envInertia + size_t(e) * m->nb * 3 : nullptr, st);
  R sumAbs = R(0);
  for (int j = 0; j < nj; ++j) sumAbs += fabs(B.prevMotor[size_t(e) * nj + j]);
  B.servoSupply[e] = rmax(R(p.vin) - R(p.vinDrop) * sumAbs, R(p.vinMin));
}

template <class R>
__global__ void bamServoJointKernel(const DevModel<R> *__restrict__ m, const R *records, int stride, int count,
                                    BamKernelParams p, BamBuffers<R> B) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const int nj = p.nj;
  if (t >= count * nj) return;
  const int e = t / nj, j = t % nj;
  const int slots = p.lag + 1;
  const R *bodies = records + size_t(e) * stride + kRecHeader;
  const int cursor = B.counters[0];
  const int delayedSlot = ((cursor - p.lag) % slots + slots) % slots;
  const size_t plane = size_t(count) * nj;
  const size_t i = size_t(e) * nj + j;
  const R target = B.home[i] + B.action[i];
  B.history[size_t(cursor) * plane + i] = target;
  if (!B.histInit[e])
    for (int s = 0; s < slots; ++s) B.history[size_t(s) * plane + i] = target;
  const R delayed = B.history[size_t(delayedSlot) * plane + i];
  R *mo = B.motor + 3 * i;
  const R ext = -mo[0] + mo[1];
  const R supply = B.servoSupply[e];
  const R kt = R(p.kt), res = R(p.res);
  const R gain = R((4096 / (2 * 3.14159265358979323846)) / (256 * 885));
  R position, velocity;
  jointState(m, bodies, j, &position, &velocity);
  const R speed = velocity;
  R duty = (delayed - position) * R(p.kpFw) * gain;
  const R center = kt * speed / supply;
  const R span = R(p.res * 1.75) / supply;
  duty = rmin(rmax(duty, center - span), center + span);
  duty = rmin(rmax(duty, R(-1)), R(1));
  const R raw = kt * supply * duty / res - R(p.kt * p.kt) * speed / res;
  const R stribeck = exp(-pow(fabs(velocity) / R(p.dthetaStribeck), R(p.alpha)));
  const R mot = B.prevApplied[i];
  const R quad = fabs(mot) > fabs(ext) ? R(p.lfeq) * (ext * ext) : R(p.lfmq) * (mot * mot);
  const R budget = R(p.fBase) + stribeck * R(p.fStribeck) + fabs(ext * R(p.lfe) - mot * R(p.lfm)) +
                   stribeck * fabs(ext * R(p.lfes) - mot * R(p.lfms)) + stribeck * quad;
  const R applied = rmin(rmax(raw, R(-p.forceLimit)), R(p.forceLimit));
  mo[0] = applied;
  mo[1] = budget;
  mo[2] = R(p.fViscous);
  B.prevMotor[i] = raw;
  B.prevApplied[i] = applied;
}

// ---------------------------------------------------------------- frames
template <class R> struct BamFrame {
  Q4<R> rq;
  V3<R> g, w, v, origin, sitePos[2], siteVel[2], footForce[2];
  bool contact[2];
};

template <class R>
__device__ __forceinline__ BamFrame<R> bamFrame(const DevModel<R> *m, const R *rec, const BamKernelParams &p,
                                                const R *rootOffset) {
  const R *bodies = rec + kRecHeader;
  const R *b1 = bodies + kRecBody;
  BamFrame<R> f;
  const Q4<R> qb{b1[3], b1[4], b1[5], b1[6]};
  f.rq = tmultiply(qb, Q4<R>{R(p.iquat[0]), R(p.iquat[1]), R(p.iquat[2]), R(p.iquat[3])});
  f.g = tinverseRotate(f.rq, V3<R>{R(0), R(0), R(-1)});
  const V3<R> wb = recV3(b1 + 10);
  f.w = tinverseRotate(f.rq, wb);
  // root_r = -inverse_rotate(q * (1, -1, -1, -1), offset)
  const V3<R> rr = tinverseRotate(Q4<R>{qb.w, -qb.x, -qb.y, -qb.z}, recV3(rootOffset));
  const V3<R> rootR{-rr.x, -rr.y, -rr.z};
  const V3<R> c = tcross(wb, rootR);
  f.origin = V3<R>{b1[7] + c.x, b1[8] + c.y, b1[9] + c.z};
  f.v = tinverseRotate(f.rq, f.origin);
  for (int k = 0; k < 2; ++k) {
    const R *fb = bodies + kRecBody * p.footBody[k];
    const Q4<R> conj{fb[3], -fb[4], -fb[5], -fb[6]};
    const V3<R> r = tinverseRotate(conj, V3<R>{R(p.site[k][0]), R(p.site[k][1]), R(p.site[k][2])});
    f.sitePos[k] = V3<R>{fb[0] + r.x, fb[1] + r.y, fb[2] + r.z};
    const V3<R> cw = tcross(recV3(fb + 10), r);
    f.siteVel[k] = V3<R>{fb[7] + cw.x, fb[8] + cw.y, fb[9] + cw.z};
    const V3<R> force = envGroundForce(m, rec, p.footBody[k]);
    f.footForce[k] = force;
    f.contact[k] = sqrt(force.x * force.x + force.y * force.y + force.z * force.z) > R(1e-5);
  }
  return f;
}

// ---------------------------------------------------------------- after substep
template <class R>
__global__ void bamAfterKernel(const DevModel<R> *__restrict__ m, const R *records, int stride, int count,
                               BamKernelParams p, BamBuffers<R> B) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= count) return;
  const R *rec = records + size_t(e) * stride;
  const R *bodies = rec + kRecHeader;
  const BamFrame<R> f = bamFrame(m, rec, p, B.rootOffset + 3 * size_t(e));
  const ContactStats<R> st = envContactStats(m, rec, true);
  B.selfContacts[e] = rmax(B.selfContacts[e], st.active);
  B.selfPenetration[e] = rmax(B.selfPenetration[e], st.depthMax);
  if (p.extras & xMeanVelocity) {
    R *mv = B.meanVelocity + 3 * size_t(e);
    const R a = R(p.meanAlpha);
    mv[0] = tlerp(mv[0], f.origin.x, a);
    mv[1] = tlerp(mv[1], f.origin.y, a);
    mv[2] = tlerp(mv[2], f.origin.z, a);
  }
  for (int k = 0; k < 2; ++k) {
    const size_t i = 2 * size_t(e) + k;
    B.contact[i] = f.contact[k];
    B.airTime[i] = f.contact[k] ? R(0) : B.airTime[i] + R(p.dt);
    B.contactTime[i] = f.contact[k] ? B.contactTime[i] + R(p.dt) : R(0);
  }
  for (int j = 0; j < p.nj; ++j) {
    R angle, rate;
    jointState(m, bodies, j, &angle, &rate);
    B.joints[(size_t(e) * p.nj + j) * 2] = angle;
    B.joints[(size_t(e) * p.nj + j) * 2 + 1] = rate;
  }
  B.histInit[e] = true;   // the servo has filled this env's delay ring
  if (e == 0) B.counters[0] = (B.counters[0] + 1) % (p.lag + 1);
}

// walking_reward.py:98-122 plus the env's overrides.
__device__ __forceinline__ void walkingWeights(const BamKernelParams &p, int iteration, double *w) {
  double action = -0.1;
  if (iteration >= 500) action = -0.2;
  if (iteration >= 750) action = -0.4;
  if (iteration >= 1000) action = -0.6;
  if (iteration >= 1250) action = -0.8;
  if (iteration >= 1500) action = -1.0;
  double head = 0.0;
  if (iteration >= 600) head = 1.0;
  if (iteration >= 1000) head = 2.0;
  if (iteration >= 1500) head = 3.0;
  const double base[15] = {2.0, 2.0, 2.0, 1.0, -0.05, -0.02, -1.0, action, 3.0, -2.0, -0.25, -0.1, -1.0, 2.0, head};
  for (int t = 0; t < 15; ++t) w[t] = (p.overrideMask >> t & 1) ? p.overrides[t] : base[t];
  w[tHeadPosition] = -p.headPosWeight;
  w[tHeadVelocity] = -p.headVelWeight;
  w[tTrackMeanVelocity] = p.meanWeight;
  w[tTrackHeading] = p.headingWeight;
}

template <class R> __device__ __forceinline__ R yawOf(Q4<R> q) {
  return atan2(R(2) * (q.w * q.z + q.x * q.y), R(1) - R(2) * (q.y * q.y + q.z * q.z));
}
template <class R> __device__ __forceinline__ R headingError(R targetYaw, Q4<R> q) {
  const R err = targetYaw - yawOf(q);
  return atan2(sin(err), cos(err));
}

// Observation rows (bam_env.py:185-211).
template <class R>
__device__ void bamWriteObs(const BamKernelParams &p, const BamBuffers<R> &B, int e, const BamFrame<R> &f) {
  const int nj = p.nj;
  float *a = B.obsActor + size_t(e) * (19 + 3 * nj);  // 3 + 3 + 3 J + 3 + 10
  float *c = B.obsCritic + size_t(e) * p.criticDim;
  const R *home = B.home + size_t(e) * nj;
  const R *jt = B.joints + size_t(e) * nj * 2;
  const R *act = B.action + size_t(e) * nj;
  const R *cmd = B.command + 3 * size_t(e);
  int o = 0;
  const V3<R> av[2] = {f.w, f.g};
  for (int k = 0; k < 2; ++k) { a[o++] = float(av[k].x); a[o++] = float(av[k].y); a[o++] = float(av[k].z); }
  for (int j = 0; j < nj; ++j) a[o++] = float(jt[2 * j] - home[j]);
  for (int j = 0; j < nj; ++j) a[o++] = float(B.observedVelocity[size_t(e) * nj + j]);
  for (int j = 0; j < nj; ++j) a[o++] = float(act[j]);
  for (int k = 0; k < 3; ++k) a[o++] = float(cmd[k]);
  for (int k = 0; k < 10; ++k) a[o++] = 0.f;
  o = 0;
  const V3<R> cv[3] = {f.v, f.w, f.g};
  for (int k = 0; k < 3; ++k) { c[o++] = float(cv[k].x); c[o++] = float(cv[k].y); c[o++] = float(cv[k].z); }
  for (int j = 0; j < nj; ++j) c[o++] = float(jt[2 * j] - home[j]);
  for (int j = 0; j < nj; ++j) c[o++] = float(jt[2 * j + 1]);
  for (int j = 0; j < nj; ++j) c[o++] = float(act[j]);
  for (int k = 0; k < 3; ++k) c[o++] = float(cmd[k]);
  c[o++] = float(f.sitePos[0].z); c[o++] = float(f.sitePos[1].z);
  c[o++] = float(B.airTime[2 * size_t(e)]); c[o++] = float(B.airTime[2 * size_t(e) + 1]);
  c[o++] = f.contact[0] ? 1.f : 0.f; c[o++] = f.contact[1] ? 1.f : 0.f;
  for (int k = 0; k < 2; ++k) {
    const R v3[3] = {f.footForce[k].x, f.footForce[k].y, f.footForce[k].z};
    for (int i = 0; i < 3; ++i) {
      const R x = v3[i];
      const R sign = x > R(0) ? R(1) : (x < R(0) ? R(-1) : R(0));
      c[o++] = float(sign * log1p(fabs(x)));
    }
  }
  for (int k = 0; k < 10; ++k) c[o++] = 0.f;
  if (p.extras & xMeanVelocity) {
    const V3<R> lm = tinverseRotate(f.rq, recV3(B.meanVelocity + 3 * size_t(e)));
    c[o++] = float(lm.x); c[o++] = float(lm.y); c[o++] = float(lm.z);
  }
  if (p.extras & xHeading) c[o++] = float(headingError(B.targetYaw[e], f.rq));
}

template <class R>
__device__ void bamStoreFrame(const BamKernelParams &p, const BamBuffers<R> &B, int e, const BamFrame<R> &f,
                              const R *rec) {
  R *x = B.features + size_t(e) * kFeatures;
  x[fFailed] = rec[0];
  x[fQuat] = f.rq.w; x[fQuat + 1] = f.rq.x; x[fQuat + 2] = f.rq.y; x[fQuat + 3] = f.rq.z;
  const V3<R> vs[4] = {f.g, f.w, f.v, f.origin};
  const int at[4] = {fGravity, fAngVel, fLinVel, fOrigin};
  for (int k = 0; k < 4; ++k) { x[at[k]] = vs[k].x; x[at[k] + 1] = vs[k].y; x[at[k] + 2] = vs[k].z; }
  for (int k = 0; k < 2; ++k) {
    x[fSitePos + 3 * k] = f.sitePos[k].x; x[fSitePos + 3 * k + 1] = f.sitePos[k].y; x[fSitePos + 3 * k + 2] = f.sitePos[k].z;
    x[fSiteVel + 3 * k] = f.siteVel[k].x; x[fSiteVel + 3 * k + 1] = f.siteVel[k].y; x[fSiteVel + 3 * k + 2] = f.siteVel[k].z;
    R *cf = B.contactForce + (2 * size_t(e) + k) * 3;
    cf[0] = f.footForce[k].x; cf[1] = f.footForce[k].y; cf[2] = f.footForce[k].z;
    B.contact[2 * size_t(e) + k] = f.contact[k];
  }
}

// ---------------------------------------------------------------- control step
// mode 0: end of a control step (bam_env.py:345-389); mode 1: refresh and
// observe after a reset (:270-275), updating the target heading of the masked
// environments and the heading command; mode 2: refresh and observe only.
template <class R>
__global__ void bamControlKernel(const DevModel<R> *__restrict__ m, const R *records, int stride, int count,
                                 BamKernelParams p, BamBuffers<R> B, int mode, const bool *mask) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= count) return;
  const int nj = p.nj;
  const R *rec = records + size_t(e) * stride;
  const R *bodies = rec + kRecHeader;
  const BamFrame<R> f = bamFrame(m, rec, p, B.rootOffset + 3 * size_t(e));
  R *jt = B.joints + size_t(e) * nj * 2;
  for (int j = 0; j < nj; ++j) jointState(m, bodies, j, &jt[2 * j], &jt[2 * j + 1]);
  bamStoreFrame(p, B, e, f, rec);
  R *cmd = B.command + 3 * size_t(e);
  if (mode != 0) {
    if (mode == 1) {
      if (mask && mask[e]) B.targetYaw[e] = yawOf(f.rq);
      if (p.headingHold) cmd[2] = rmin(rmax(R(0.5) * headingError(B.targetYaw[e], f.rq), R(-1)), R(1));
    }
    bamWriteObs(p, B, e, f);
    return;
  }
  const long long len = B.episodeLength[e] + 1;
  B.episodeLength[e] = len;
  const R *home = B.home + size_t(e) * nj;
  const R *act = B.action + size_t(e) * nj;
  const R *old = B.oldAction + size_t(e) * nj;
  if (p.reward) {
    R terms[kBamTerms];
    for (int t = 0; t < kBamTerms; ++t) terms[t] = R(0);
    const R speed = sqrt(cmd[0] * cmd[0] + cmd[1] * cmd[1]) + fabs(cmd[2]);
    const R active = speed > R(0.01) ? R(1) : R(0);
    const bool standing = speed < R(0.01);
    // Swing peaks and the first-contact mask.
    R *peak = B.peakHeight + 2 * size_t(e);
    R swing = R(0), clearance = R(0), slip = R(0), air = R(0);
    for (int k = 0; k < 2; ++k) {
      const R ct = B.contactTime[2 * size_t(e) + k], at = B.airTime[2 * size_t(e) + k];
      const bool first = ct > R(0) && ct < R(p.stepDt + 1e-8);
      const R height = f.sitePos[k].z;
      if (!f.contact[k]) peak[k] = rmax(peak[k], height);
      const R d = peak[k] / R(0.02) - R(1);
      swing += first ? d * d : R(0);
      if (first) peak[k] = R(0);
      const R fs2 = f.siteVel[k].x * f.siteVel[k].x + f.siteVel[k].y * f.siteVel[k].y;
      clearance += fabs(height - R(0.02)) * sqrt(fs2);
      slip += f.contact[k] ? fs2 : R(0);
      air += (at > R(0.125) && at < R(0.3)) ? R(1) : R(0);
    }
    terms[tFootSwing] = swing * active;
    terms[tFootClearance] = clearance * active;
    terms[tFootSlip] = slip * active;
    terms[tAirTime] = air * active;
    // Head moving average and pose terms.
    R *ema = B.headEma + 4 * size_t(e);
    const R alpha = R(p.stepDt < 1.0 ? p.stepDt : 1.0);
    R pose = R(0), headTrack = R(0), headBias = R(0), headPos = R(0), headVel = R(0), limits = R(0), rate = R(0);
    int legs = 0, heads = 0;
    for (int j = 0; j < nj; ++j) {
      const R q = jt[2 * j], err = q - home[j];
      limits += rmax(R(p.soft[j][0]) - q, R(0)) + rmax(q - R(p.soft[j][1]), R(0));
      const R da = act[j] - old[j];
      rate += da * da;
      if (p.headMask >> j & 1) {
        R h = len <= 1 ? R(0) : ema[heads];
        h = (R(1) - alpha) * h + alpha * err;
        ema[heads] = h;
        const R z = err / R(0.5);
        headTrack += exp(-(z * z));
        headBias += fabs(h);
        headPos += err * err;
        headVel += jt[2 * j + 1] * jt[2 * j + 1];
        ++heads;
      } else {
        const R z = err / R(standing ? p.stand[j] : p.walk[j]);
        pose += z * z;
        ++legs;
      }
    }
    const R dvx = f.v.x - cmd[0], dvy = f.v.y - cmd[1];
    terms[tTrackLin] = exp(-(dvx * dvx + dvy * dvy) / R(p.linVar) - f.v.z * f.v.z / R(p.vertVar));
    const R dwz = f.w.z - cmd[2];
    terms[tTrackAng] = exp(-(dwz * dwz + (f.w.x * f.w.x + f.w.y * f.w.y)) / R(0.5));
    terms[tUpright] = exp(-(f.g.x * f.g.x + f.g.y * f.g.y) / R(0.05));
    terms[tPose] = exp(-(pose / R(legs)));
    const R *b1 = bodies + kRecBody;
    terms[tBodyAngVel] = b1[10] * b1[10] + b1[11] * b1[11];
    // Angular momentum about the centre of mass (bam_env.py:419-428).
    V3<R> com{R(0), R(0), R(0)};
    R total = R(0);
    for (int b = 0; b < m->nb; ++b) {
      const R mb = __ldg(&m->mass[b]);
      const R *bb = bodies + kRecBody * b;
      com = com + recV3(bb) * mb;
      total += mb;
    }
    com = com * (R(1) / total);
    V3<R> L{R(0), R(0), R(0)};
    for (int b = 0; b < m->nb; ++b) {
      const R mb = __ldg(&m->mass[b]);
      const R *bb = bodies + kRecBody * b;
      const Q4<R> q{bb[3], bb[4], bb[5], bb[6]};
      const V3<R> lw = rotateInv(q, recV3(bb + 10));
      const V3<R> in = mvec(m->inertia[b]);
      const V3<R> spin = rotate(q, V3<R>{in.x * lw.x, in.y * lw.y, in.z * lw.z});
      L = L + spin + cross(recV3(bb) - com, recV3(bb + 7) * mb);
    }
    terms[tAngMomentum] = dot(L, L);
    terms[tDofLimits] = limits;
    terms[tActionRate] = rate;
    terms[tSelfCollisions] = B.selfContacts[e];
    terms[tHeadTracking] = headTrack / R(heads);
    terms[tHeadBias] = -(headBias / R(heads));
    terms[tHeadPosition] = headPos;
    terms[tHeadVelocity] = headVel;
    if (p.extras & xMeanVelocity) {
      const V3<R> lm = tinverseRotate(f.rq, recV3(B.meanVelocity + 3 * size_t(e)));
      const R mx = lm.x - cmd[0], my = lm.y - cmd[1];
      terms[tTrackMeanVelocity] = exp(-(mx * mx + my * my) / R(p.meanVar));
    }
    if (p.extras & xHeading) {
      const R he = headingError(B.targetYaw[e], f.rq);
      terms[tTrackHeading] = exp(-(he * he) / R(p.headingVar));
    }
    double w[kBamTerms];
    walkingWeights(p, p.sourceIteration + B.counters[1] / 24, w);
    R r = R(0);
    for (int t = 0; t < kBamTerms; ++t) {
      const bool on = t < 15 || ((t == tHeadPosition || t == tHeadVelocity) && (p.extras & xHeadStability)) ||
                      (t == tTrackMeanVelocity && (p.extras & xMeanVelocity)) ||
                      (t == tTrackHeading && (p.extras & xHeading));
      if (on) r += R(w[t]) * terms[t];
      B.terms[size_t(e) * kBamTerms + t] = terms[t];
    }
    B.reward[e] = float(r * R(p.stepDt));
  } else {
    B.reward[e] = 0.f;
  }
  const bool timeout = len >= p.maxEpisode;
  bool finite = true;
  for (int j = 0; j < 2 * nj; ++j) finite &= isfinite(jt[j]);
  const bool failed = f.g.z > R(p.tiltLimit) || rec[0] > R(0) || rec[2] > R(0.005) || rec[3] > R(0.005) ||
                      B.selfPenetration[e] > R(0.005) || !finite;
  B.timeout[e] = timeout;
  B.failed[e] = failed;
  B.done[e] = timeout || failed;
  if (p.headingHold) cmd[2] = rmin(rmax(R(0.5) * headingError(B.targetYaw[e], f.rq), R(-1)), R(1));
  bamWriteObs(p, B, e, f);
}

// ---------------------------------------------------------------- reset
// bam_env.py:245-275 (the buffer part; noise, commands and the physics reset
// are issued by the host).
template <class R>
__global__ void bamResetKernel(BamKernelParams p, BamBuffers<R> B, int count, const bool *mask) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= count || !mask[e]) return;
  const int nj = p.nj, slots = p.lag + 1;
  const size_t plane = size_t(count) * nj;
  for (int j = 0; j < nj; ++j) {
    const size_t i = size_t(e) * nj + j;
    B.action[i] = B.oldAction[i] = B.prevMotor[i] = B.prevApplied[i] = B.observedVelocity[i] = R(0);
    for (int s = 0; s < slots; ++s) B.history[size_t(s) * plane + i] = B.home[i];
  }
  for (int k = 0; k < 2; ++k) {
    B.airTime[2 * size_t(e) + k] = B.contactTime[2 * size_t(e) + k] = R(0);
    B.peakHeight[2 * size_t(e) + k] = R(0);
  }
  for (int k = 0; k < 3; ++k) B.meanVelocity[3 * size_t(e) + k] = R(0);
  for (int k = 0; k < 4; ++k) B.headEma[4 * size_t(e) + k] = R(0);
  B.selfContacts[e] = B.selfPenetration[e] = R(0);
  B.episodeLength[e] = 0;
  B.histInit[e] = false;
}

}  // namespace duckb200
