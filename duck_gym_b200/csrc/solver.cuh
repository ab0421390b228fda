// The AVBD environment step on sm_100a: one team of T lanes per environment
// (T = 8 for the biped, four environments per warp), every environment's
// working state kept in shared memory for all substeps of a call.
//
// Algorithm: the reference's BasicState::advance / step (src/cuda/kernel.cuh:
// 421-443, 937-1095) -- contact generation, joint warm start and predictor,
// colored Gauss-Seidel block solves, augmented-Lagrangian dual and penalty
// updates with the friction-cone clamp, velocity recovery and diagnostics.
// What differs is the mapping onto the GPU:
//  * the reference runs one 32-lane warp per environment and executes the
//    warm start, predictor, contact construction and velocity recovery on
//    lane 0; here every phase is spread over the team (a lane per body, joint,
//    shape or contact), and 4 environments share a warp;
//  * each body keeps its rotation matrix on chip, so every hinge and contact
//    lever is a 9-FMA product; each body also keeps a bit mask of the contacts
//    that touch it;
//  * the primal update of a body exploits the structure of each Jacobian row
//    (unit-axis linear rows, pure angular rows), forms the geometric-stiffness
//    majorizer of the unit-axis rows in closed form, assembles only the lower
//    triangle of the 6x6 block, and sums every hinge-axis term (limits, PD
//    drive, damping, dry friction) into one rank-one update;
//  * the frozen world inertia of a body is formed once per substep;
//  * the four environments of a warp are interleaved word by word in shared
//    memory (element i of team t at word 4 i + t) and every per-body and
//    per-contact stride is odd, so lanes of different teams never share a
//    bank and lanes of one team rarely do;
//  * contact generation reproduces the reference's arithmetic bit for bit
//    (x-prefixed ops of dmath.cuh) so contact sets match the CPU exactly.
#pragma once
#include "dmath.cuh"
#include "model.hpp"

namespace duckb200 {

// Portable record: header 8, bodies B x 16, joints J x 22, contacts bound x 32.
constexpr int kRecHeader = 8, kRecBody = 16, kRecJoint = 22, kRecContact = 32;
// On-chip contact entry (17 words, odd for conflict-free lane-strided
// access): packed keys, feature, local(3), anchor or localB(3), friction, c0,
// lambda(3), penalty(3), padding.
constexpr int kC = 17;
enum { cMeta = 0, cFeature = 1, cLocal = 2, cAnchor = 5, cFriction = 8, cC0 = 9, cLambda = 10, cPenalty = 13 };
// Team-shared integers.
enum { iFailed = 0, iCount = 1, iGround = 2, iColors = 3, iPrevCount = 4, iMisc = 8 };

// Strides of the per-body arrays (odd: see the interleaving note above).
constexpr int kSQ = 5, kSIW = 7;

struct Layout {
  int X, Q, RM, XQP, IW, F1;                           // bodies (XQP: v,w between substeps, x~,q~ inside)
  int JL, JP, JC0, JA0, JV0, JLF, JPF, JT, JTQ, JFL, JD;  // joints
  int C, CB;                                           // contacts, self-contact basis
  int I;                                               // ints (Real slot offset)
  int colors, colorList, colorStart, masks, prevKeys;  // offsets inside the int region
  int cap, pairCap, maxColors;
  int size;                                            // Reals per environment
};

template <class R> __host__ inline Layout makeLayout(const DevModel<R> &m) {
  Layout L{};
  int o = 0;
  auto take = [&](int n) { int at = o; o += n; return at; };
  const int nb = m.nb, nj = m.nj;
  L.X = take(3 * nb); L.Q = take(kSQ * nb); L.RM = take(9 * nb); L.XQP = take(7 * nb);
  L.IW = take(kSIW * nb); L.F1 = take(3);
  L.JL = take(7 * nj); L.JP = take(7 * nj); L.JC0 = take(7 * nj); L.JA0 = take(nj);
  L.JV0 = take(nj); L.JLF = take(nj); L.JPF = take(nj); L.JT = take(nj); L.JTQ = take(nj);
  L.JFL = take(nj); L.JD = take(nj);
  L.cap = m.groundCap + m.np;
  L.pairCap = m.np;
  L.C = take(kC * std::max(L.cap, 1));
  L.CB = take(9 * std::max(L.pairCap, 1));
  L.maxColors = 2 + m.np;
  L.colors = iMisc;
  L.colorList = iMisc + nb;
  L.colorStart = iMisc + 2 * nb;
  L.masks = L.colorStart + L.maxColors + 1;
  // Ground keys of the previous substep's contacts (warm-start lookup).
  L.prevKeys = L.masks + 2 * nb;
  // One Real slot per integer keeps the interleaved addressing uniform.
  L.I = take(L.prevKeys + std::max(L.cap, 1));
  L.size = o;
  return L;
}

template <class T> __device__ __forceinline__ T ldg(const T &v) { return __ldg(&v); }

// A team's view of the interleaved shared block: element i at p[i * STRIDE].
template <class R, int STRIDE> struct View {
  R *p;
  __device__ __forceinline__ R &operator[](int i) const { return p[i * STRIDE]; }
  __device__ __forceinline__ View operator+(int i) const { return {p + i * STRIDE}; }
};
template <class R, int STRIDE> struct IntView {
  R *p;
  __device__ __forceinline__ int &operator[](int i) const { return reinterpret_cast<int &>(p[i * STRIDE]); }
};

template <int T> struct Team {
  unsigned mask;
  int lane;
  __device__ __forceinline__ Team() {
    int l = threadIdx.x & 31;
    lane = l & (T - 1);
    mask = T == 32 ? 0xffffffffu : (((1u << T) - 1u) << (l & ~(T - 1)));
  }
  __device__ __forceinline__ void sync() const { __syncwarp(mask); }
  template <class V> __device__ __forceinline__ V max(V v) const {
#pragma unroll
    for (int o = T / 2; o > 0; o >>= 1) {
      V u = __shfl_xor_sync(mask, v, o, T);
      v = v > u ? v : u;
    }
    return v;
  }
  __device__ __forceinline__ bool any(bool p) const { return __any_sync(mask, p); }
  // Exclusive prefix sum over the team; *total receives the team sum.
  __device__ __forceinline__ int scan(int v, int *total) const {
    int x = v;
#pragma unroll
    for (int o = 1; o < T; o <<= 1) {
      int y = __shfl_up_sync(mask, x, o, T);
      if (lane >= o) x += y;
    }
    *total = __shfl_sync(mask, x, T - 1, T);
    return x - v;
  }
};

struct StepArgs {
  const void *target;   // [E,J] (step) or nullptr
  const void *forces;   // [E,3]
  const void *motor;    // [E,J,3] (step_motor) or nullptr
  int substeps;
  double kp, limit;
  // Per-environment physical parameters (domain randomisation, an extension
  // beyond the reference's shared model), nullptr = the model's values:
  // body masses [E,B], principal inertias [E,B,3], shape frictions [E,S].
  const void *mass = nullptr, *inertia = nullptr, *friction = nullptr;
};

// P = false: a model without body-collision pairs (its colours never change
// and every contact is a ground contact); the body-pair code is compiled out
// of that instantiation.
template <class R, int T, bool P = true> struct Solver {
  __device__ __forceinline__ bool pairs() const { return P && m->np > 0; }
  static constexpr int kTeams = 32 / T;
  static constexpr int kPerLane = (kMaxBodies + T - 1) / T;   // bodies per lane in lane-per-body loops
  // Lanes that share one body's block update in the Gauss-Seidel sweep: with
  // 16 or more lanes per environment a colour's bodies outnumber half the
  // team at most, so each body gets two lanes that split its rows.
  static constexpr int kSplit = T >= 16 ? 2 : 1;
  using SV = View<R, kTeams>;
  const DevModel<R> *__restrict__ m;
  const R *__restrict__ pts;
  SV S;                    // environment's interleaved shared-memory view
  IntView<R, kTeams> I;    // its integer region
  R *rec;                  // environment's global record
  const Layout &L;
  Team<T> team;
  // This environment's randomised parameters (nullptr: the model's).
  const R *envMass = nullptr, *envInertia = nullptr, *envFriction = nullptr;
  // 1 / dt and its square, divided once per launch (the compiler does not
  // hoist the division out of the stamp loops on its own), and the model's
  // solver constants, read once into registers instead of from the model in
  // every stamp and dual update.
  R ih, ih2;
  R sDt, sAlpha, sGamma, sBetaL, sBetaA;

  __device__ Solver(const DevModel<R> *model, const R *points, R *smemTeam, R *record, const Layout &layout)
      : m(model), pts(points), S{smemTeam}, rec(record), L(layout) {
    I = IntView<R, kTeams>{smemTeam + size_t(L.I) * kTeams};
    ih = R(1) / m->dt;
    sDt = m->dt;
    sAlpha = m->alpha;
    sGamma = m->gamma;
    sBetaL = m->betaLinear;
    sBetaA = m->betaAngular;
    ih2 = ih * ih;
  }

  // ------------------------------------------------------------ accessors
  __device__ __forceinline__ V3<R> ld3(int off) const { return {S[off], S[off + 1], S[off + 2]}; }
  __device__ __forceinline__ Q4<R> ld4(int off) const { return {S[off], S[off + 1], S[off + 2], S[off + 3]}; }
  __device__ __forceinline__ void st3(int off, V3<R> v) { S[off] = v.x; S[off + 1] = v.y; S[off + 2] = v.z; }
  __device__ __forceinline__ void st4(int off, Q4<R> q) { S[off] = q.w; S[off + 1] = q.x; S[off + 2] = q.y; S[off + 3] = q.z; }
  __device__ __forceinline__ V3<R> mv3(const R (&a)[3]) const { return {ldg(a[0]), ldg(a[1]), ldg(a[2])}; }
  __device__ __forceinline__ Q4<R> mq4(const R (&a)[4]) const { return {ldg(a[0]), ldg(a[1]), ldg(a[2]), ldg(a[3])}; }
  __device__ __forceinline__ SV rot(int b) const { return S + (L.RM + 9 * b); }
  __device__ __forceinline__ Q4<R> quat(int b) const { return ld4(L.Q + kSQ * b); }
  __device__ __forceinline__ void setPose(int b, V3<R> x, Q4<R> q) {
    st3(L.X + 3 * b, x);
    st4(L.Q + kSQ * b, q);
    R mm[9];
    quatToMatrix(q, mm);
#pragma unroll
    for (int k = 0; k < 9; ++k) S[L.RM + 9 * b + k] = mm[k];
  }
  // Mass, principal inertia and ground friction of this environment: the
  // model's, or the randomised values for dynamic bodies.
  __device__ __forceinline__ R massOf(int b) const {
    const R mm = ldg(m->mass[b]);
    return envMass && mm > R(0) ? envMass[b] : mm;
  }
  __device__ __forceinline__ V3<R> inertiaOf(int b) const {
    return envInertia && ldg(m->mass[b]) > R(0) ? V3<R>{envInertia[3 * b], envInertia[3 * b + 1], envInertia[3 * b + 2]}
                                                : mv3(m->inertia[b]);
  }
  __device__ __forceinline__ R frictionOf(int s) const { return envFriction ? envFriction[s] : ldg(m->sFriction[s]); }
  // Velocities live in the XQP slots between substeps (predicted poses inside).
  __device__ __forceinline__ V3<R> vel(int b) const { return ld3(L.XQP + 7 * b); }
  __device__ __forceinline__ V3<R> omega(int b) const { return ld3(L.XQP + 7 * b + 3); }
  __device__ __forceinline__ V3<R> bodyForce(int b) const {
    return b == 1 ? ld3(L.F1) : V3<R>{R(0), R(0), R(0)};
  }
  __device__ __forceinline__ SV contact(int c) const { return S + (L.C + kC * c); }
  __device__ __forceinline__ int &cmeta(int c) const { return reinterpret_cast<int &>(S[L.C + kC * c + cMeta]); }

  __device__ __forceinline__ int &cfeat(int c) const { return reinterpret_cast<int &>(S[L.C + kC * c + cFeature]); }
  // meta: body (5 bits) | other + 1 (6) | stick (1) | shape (5) | otherShape + 1 (6)
  __device__ static __forceinline__ int packMeta(int body, int other, int shape, int otherShape) {
    return body | ((other + 1) << 5) | (shape << 12) | ((otherShape + 1) << 17);
  }
  __device__ static __forceinline__ int metaBody(int meta) { return meta & 31; }
  __device__ static __forceinline__ int metaOther(int meta) { return ((meta >> 5) & 63) - 1; }
  __device__ static __forceinline__ bool metaStick(int meta) { return (meta >> 11) & 1; }
  __device__ static __forceinline__ int metaShape(int meta) { return (meta >> 12) & 31; }
  __device__ static __forceinline__ int metaOtherShape(int meta) { return ((meta >> 17) & 63) - 1; }

  // ------------------------------------------------------------ load / store
  // Record -> shared memory.  Contacts stay in the record: the first
  // substep's warm start reads them from there.
  __device__ void load() {
    const int nb = m->nb, nj = m->nj;
    for (int b = team.lane; b < nb; b += T) {
      const R *r = rec + kRecHeader + kRecBody * b;
      setPose(b, {r[0], r[1], r[2]}, {r[3], r[4], r[5], r[6]});
      SV vw = S + (L.XQP + 7 * b);
      vw[0] = r[7]; vw[1] = r[8]; vw[2] = r[9]; vw[3] = r[10]; vw[4] = r[11]; vw[5] = r[12];
    }
    for (int j = team.lane; j < nj; j += T) {
      const R *r = rec + kRecHeader + kRecBody * nb + kRecJoint * j;
#pragma unroll
      for (int k = 0; k < 7; ++k) {
        S[L.JL + 7 * j + k] = r[k];
        S[L.JP + 7 * j + k] = r[7 + k];
      }
      S[L.JLF + j] = r[14];
      S[L.JPF + j] = r[15];
      S[L.JT + j] = r[16];
      S[L.JTQ + j] = r[19];
      S[L.JFL + j] = r[20];
      S[L.JD + j] = r[21];
    }
    if (team.lane == 0) {
      const R *r = rec + kRecHeader + kRecBody * 1;
      st3(L.F1, {r[13], r[14], r[15]});
      I[iFailed] = int(rec[0]);
      I[iPrevCount] = int(rec[1]);
      I[iCount] = 0;
    }
  }
  // Shared memory -> record (bodies, joints); contacts are written at the
  // end of every substep and the header by storeHeader.
  __device__ void store(R kp, R limit) {
    const int nb = m->nb, nj = m->nj;
    for (int b = team.lane; b < nb; b += T) {
      R *r = rec + kRecHeader + kRecBody * b;
      V3<R> x = ld3(L.X + 3 * b), v = vel(b), w = omega(b);
      Q4<R> q = quat(b);
      r[0] = x.x; r[1] = x.y; r[2] = x.z; r[3] = q.w; r[4] = q.x; r[5] = q.y; r[6] = q.z;
      r[7] = v.x; r[8] = v.y; r[9] = v.z; r[10] = w.x; r[11] = w.y; r[12] = w.z;
      if (b == 1) { V3<R> f = ld3(L.F1); r[13] = f.x; r[14] = f.y; r[15] = f.z; }
    }
    for (int j = team.lane; j < nj; j += T) {
      R *r = rec + kRecHeader + kRecBody * nb + kRecJoint * j;
#pragma unroll
      for (int k = 0; k < 7; ++k) {
        r[k] = S[L.JL + 7 * j + k];
        r[7 + k] = S[L.JP + 7 * j + k];
      }
      r[14] = S[L.JLF + j]; r[15] = S[L.JPF + j]; r[16] = S[L.JT + j]; r[17] = kp;
      r[18] = limit; r[19] = S[L.JTQ + j]; r[20] = S[L.JFL + j]; r[21] = S[L.JD + j];
    }
  }
  __device__ void storeHeader(R jointError, R penetration, int contacts, bool converged, R axisError,
                              int iterations) {
    if (team.lane == 0) {
      rec[0] = R(I[iFailed]);
      rec[2] = jointError; rec[3] = penetration; rec[4] = R(contacts); rec[5] = R(converged);
      rec[6] = axisError; rec[7] = R(iterations);
    }
  }
  // On-chip contact list -> record (the warm-start cache of the next substep).
  __device__ void storeContacts() {
    const int n = I[iCount], nGround = I[iGround];
    R *base = rec + kRecHeader + kRecBody * m->nb + kRecJoint * m->nj;
    for (int c = team.lane; c < n; c += T) {
      const SV s = contact(c);
      R *r = base + kRecContact * c;
      const int meta = cmeta(c);
      const int other = metaOther(meta);
      r[0] = R(metaBody(meta)); r[1] = R(metaShape(meta)); r[2] = R(cfeat(c)); r[3] = R(other);
      r[4] = R(metaOtherShape(meta)); r[5] = R(metaStick(meta) ? 1 : 0);
      r[6] = s[cLocal]; r[7] = s[cLocal + 1]; r[8] = s[cLocal + 2];
      if (!P || other < 0) {
        r[9] = s[cAnchor]; r[10] = s[cAnchor + 1]; r[11] = s[cAnchor + 2];
        r[12] = r[13] = r[14] = R(0);
        r[15] = R(1); r[16] = R(0); r[17] = R(0); r[18] = R(0); r[19] = R(1); r[20] = R(0);
        r[21] = R(0); r[22] = R(0); r[23] = R(1);
      } else {
        const SV bs = S + (L.CB + 9 * (c - nGround));
        r[9] = r[10] = r[11] = R(0);
        r[12] = s[cAnchor]; r[13] = s[cAnchor + 1]; r[14] = s[cAnchor + 2];
#pragma unroll
        for (int k = 0; k < 9; ++k) r[15 + k] = bs[k];
      }
      r[24] = s[cFriction]; r[25] = s[cC0];
#pragma unroll
      for (int k = 0; k < 3; ++k) { r[26 + k] = s[cLambda + k]; r[29 + k] = s[cPenalty + k]; }
    }
    if (team.lane == 0) rec[1] = R(n);
  }

  // ------------------------------------------------------------ contacts
  // Support point k of a ground shape in body coordinates (kernel.cuh:576-583).
  __device__ V3<R> xpoint(int s, Q4<R> q, int k) const {
    int type = ldg(m->sType[s]);
    if (type == 1 || type == 3) {
      const R *p = pts + 3 * (ldg(m->sOffset[s]) + k);
      return {ldg(p[0]), ldg(p[1]), ldg(p[2])};
    }
    V3<R> size = mv3(m->sSize[s]), center = mv3(m->sCenter[s]);
    V3<R> down = xrotate(conj(q), V3<R>{R(0), R(0), -size.x});
    if (type == 0) return xadd(center, down);
    V3<R> off = xrotate(mq4(m->sQ[s]), V3<R>{R(0), R(0), xmul(R(k ? 1 : -1), size.y)});
    return xadd(xadd(center, off), down);
  }
  // World point k of shape s and its predicted height (kernel.cuh:614-630).
  __device__ __forceinline__ R pickPoint(int s, int k, V3<R> x, V3<R> v, V3<R> w, Q4<R> q, R dt, R dt2, R accel,
                                         V3<R> &wp) const {
    V3<R> local = xpoint(s, q, k);
    wp = xadd(x, xrotate(q, local));
    V3<R> vv = xadd(v, xcross(w, xsub(wp, x)));
    return rmin(wp.z, xadd(xadd(wp.z, xmul(dt, vv.z)), xmul(dt2, accel)));
  }
  // The reference's lateral test hypot(dx, dy) < .005 (kernel.cuh:355):
  // its float hypot is correctly rounded and the comparison is in double.
  // The root and both roundings are monotone in s = dx^2 + dy^2 (exact
  // squares, summed in double), so the test is s < kPickApart2, the least
  // double whose rounded root narrows to a float >= .005.  The constant is
  // found by bisection over the doubles (tests/test_pick_threshold.py derives
  // it again); this replaces a double square root per test.
  static constexpr double kPickApart2 = 0x1.a36e30068db92p-16;
  static __device__ __forceinline__ bool pickClose(float dx, float dy) {
    const double x = dx, y = dy;
    return __dadd_rn(__dmul_rn(x, x), __dmul_rn(y, y)) < kPickApart2;
  }
  static __device__ __forceinline__ bool pickClose(double dx, double dy) { return xhypot(dx, dy) < .005; }
  // A candidate pick must lie 5 mm or more (laterally) from the earlier ones.
  static __device__ __forceinline__ bool pickApart(V3<R> wp, const V3<R> *world, int n) {
    bool ok = true;
#pragma unroll
    for (int c = 0; c < 3; ++c)
      if (c < n && pickClose(xsub(world[c].x, wp.x), xsub(world[c].y, wp.y))) ok = false;
    return ok;
  }
  // Up to four lowest, laterally separated support points of shape s that are
  // predicted below 3 mm (kernel.cuh:338-364, 601-653), on one lane.
  __device__ __forceinline__ int groundPicks(int s, int *feature, V3<R> *world) const {
    const int b = ldg(m->sBody[s]);
    const R mass = massOf(b);
    if (!m->ground || !ldg(m->sGround[s]) || mass == R(0)) return 0;
    const R dt = m->dt;
    V3<R> x = ld3(L.X + 3 * b), v = vel(b), w = omega(b);
    Q4<R> q = quat(b);
    const R accel = xadd(m->gravity[2], bodyForce(b).z / mass);
    const R dt2 = xmul(dt, dt);
    R low = rmin(x.z, xadd(xadd(x.z, xmul(dt, v.z)), xmul(dt2, accel)));
    if (double(xsub(low, xmul(ldg(m->sRadius[s]), xadd(R(1), xmul(dt, xnorm(w)))))) >= .003) return 0;
    const int count = ldg(m->sCount[s]);
    int n = 0;
    // Up to 4 picks of the lowest predicted points below 3 mm, 5 mm apart
    // laterally.  Shapes of at most 8 points (spheres, capsules, boxes) keep
    // their world points and predicted heights in registers across the picks;
    // larger point sets recompute them per pick.  Either way every point is
    // evaluated with the same arithmetic, so the picks are identical.
    if (count <= 8) {
      // The candidates still open for a pick: below 3 mm and 5 mm or more
      // (laterally) from every earlier pick.  After each pick the distance test
      // runs for all candidates at once (independent, so it pipelines) instead
      // of inside the scan; the scan keeps the reference's order and
      // comparisons (first candidate not above the running minimum), NaN
      // heights included, so the picks are the same.
      V3<R> wps[8];
      R zs[8];
      unsigned open = 0u;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (k < count) {
          zs[k] = pickPoint(s, k, x, v, w, q, dt, dt2, accel, wps[k]);
          if (!(double(zs[k]) >= .003)) open |= 1u << k;
        }
      for (int pick = 0; pick < 4 && open; ++pick) {
        int best = -1;
        R lowest = R(INFINITY);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if ((open >> k & 1u) && !(zs[k] >= lowest)) {
            best = k;
            lowest = zs[k];
          }
        if (best < 0) break;
        V3<R> bestWorld{};
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (k == best) bestWorld = wps[k];
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (c == n) { feature[c] = best; world[c] = bestWorld; }
        ++n;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if ((open >> k & 1u) && pickClose(xsub(bestWorld.x, wps[k].x), xsub(bestWorld.y, wps[k].y)))
            open &= ~(1u << k);
      }
      return n;
    }
    for (int pick = 0; pick < 4; ++pick) {
      int best = -1;
      R lowest = R(INFINITY);
      V3<R> bestWorld{};
      for (int k = 0; k < count; ++k) {
        V3<R> wp;
        const R z = pickPoint(s, k, x, v, w, q, dt, dt2, accel, wp);
        if (double(z) >= .003 || z >= lowest || !pickApart(wp, world, n)) continue;
        best = k;
        lowest = z;
        bestWorld = wp;
      }
      if (best < 0) break;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (c == n) { feature[c] = best; world[c] = bestWorld; }
      ++n;
    }
    return n;
  }
  // Warm-start data of a previous ground contact, read from the record.
  struct WarmStart {
    R lambda[3], penalty[3];
    V3<R> local, anchor;
    bool found, stick;
  };
  // Ground contact with warm start (kernel.cuh:618-650).
  __device__ __forceinline__ void buildGround(int slot, int s, int best, V3<R> bestWorld, const WarmStart &w) {
    const int b = ldg(m->sBody[s]);
    V3<R> x = ld3(L.X + 3 * b);
    Q4<R> q = quat(b);
    V3<R> local = xpoint(s, q, best);
    V3<R> anchor{bestWorld.x, bestWorld.y, R(0)};
    R lambda[3] = {R(0), R(0), R(0)}, penalty[3] = {R(1000), R(1000), R(1000)};
    if (w.found) {
#pragma unroll
      for (int d = 0; d < 3; ++d) { lambda[d] = w.lambda[d]; penalty[d] = w.penalty[d]; }
      if (w.stick) {
        local = w.local;
        anchor = w.anchor;
      }
    }
    const R c0 = rmin(xadd(x, xrotate(q, local)).z, R(0));
    const R ag = xmul(m->alpha, m->gamma);
    SV c = contact(slot);
    cmeta(slot) = packMeta(b, -1, s, -1);
    cfeat(slot) = best;
    c[cLocal] = local.x; c[cLocal + 1] = local.y; c[cLocal + 2] = local.z;
    c[cAnchor] = anchor.x; c[cAnchor + 1] = anchor.y; c[cAnchor + 2] = anchor.z;
    c[cFriction] = frictionOf(s);
    c[cC0] = c0;
#pragma unroll
    for (int d = 0; d < 3; ++d) {
      c[cLambda + d] = xmul(lambda[d], ag);
      c[cPenalty + d] = rclamp(xmul(penalty[d], m->gamma), R(1000), R(1e9));
    }
  }
  // Warm-start entry of a pick: the first previous contact with the same
  // shape and feature, read from the record.
  __device__ __forceinline__ WarmStart warmStart(int match) const {
    WarmStart w;
    w.found = match >= 0;
    if (w.found) {
      const R *p = rec + kRecHeader + kRecBody * m->nb + kRecJoint * m->nj + kRecContact * match;
#pragma unroll
      for (int d = 0; d < 3; ++d) { w.lambda[d] = p[26 + d]; w.penalty[d] = p[29 + d]; }
      w.stick = p[5] != R(0);
      w.local = {p[6], p[7], p[8]};
      w.anchor = {p[9], p[10], p[11]};
    }
    return w;
  }
  // The ground contacts of one shape's n picks.  Without body pairs the
  // warm-start entries of all picks are looked up first and their record
  // reads issued together, so the picks wait for one round trip to the
  // record instead of one each; the pair instantiation, short of registers,
  // keeps one pick at a time.
  __device__ __forceinline__ void buildGroundPicks(int s, int n, const int (&feature)[4], const V3<R> (&world)[4],
                                                   int first, int prevCount) {
    if constexpr (!P) {
      int key[4], match[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        key[k] = k < n ? groundKey(s, feature[k]) : -2;
        match[k] = -1;
      }
      for (int i = 0; i < prevCount; ++i) {
        const int have = I[L.prevKeys + i];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (match[k] < 0 && have == key[k]) match[k] = i;
      }
      WarmStart w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) w[k] = warmStart(match[k]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (k >= n) break;
        const int slot = first + k;
        if (slot < L.cap) buildGround(slot, s, feature[k], world[k], w[k]);
        else I[iFailed] = 1;
      }
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (k >= n) break;
        const int slot = first + k;
        if (slot < L.cap) buildGroundSearch(slot, s, feature[k], world[k], prevCount);
        else I[iFailed] = 1;
      }
    }
  }

  // Ground contact with warm start from the record, searched and read for
  // one pick at a time (kernel.cuh:618-650): the pair instantiation.
  __device__ void buildGroundSearch(int slot, int s, int best, V3<R> bestWorld, int prevCount) {
    const int b = ldg(m->sBody[s]);
    V3<R> x = ld3(L.X + 3 * b);
    Q4<R> q = quat(b);
    V3<R> local = xpoint(s, q, best);
    V3<R> anchor{bestWorld.x, bestWorld.y, R(0)};
    R lambda[3] = {R(0), R(0), R(0)}, penalty[3] = {R(1000), R(1000), R(1000)};
    const R *prev = rec + kRecHeader + kRecBody * m->nb + kRecJoint * m->nj;
    const int key = groundKey(s, best);
    for (int i = 0; i < prevCount; ++i) {
      if (I[L.prevKeys + i] == key) {
        const R *p = prev + kRecContact * i;
#pragma unroll
        for (int d = 0; d < 3; ++d) { lambda[d] = p[26 + d]; penalty[d] = p[29 + d]; }
        if (p[5] != R(0)) {
          local = {p[6], p[7], p[8]};
          anchor = {p[9], p[10], p[11]};
        }
        break;
      }
    }
    const R c0 = rmin(xadd(x, xrotate(q, local)).z, R(0));
    const R ag = xmul(m->alpha, m->gamma);
    SV c = contact(slot);
    cmeta(slot) = packMeta(b, -1, s, -1);
    cfeat(slot) = best;
    c[cLocal] = local.x; c[cLocal + 1] = local.y; c[cLocal + 2] = local.z;
    c[cAnchor] = anchor.x; c[cAnchor + 1] = anchor.y; c[cAnchor + 2] = anchor.z;
    c[cFriction] = frictionOf(s);
    c[cC0] = c0;
#pragma unroll
    for (int d = 0; d < 3; ++d) {
      c[cLambda + d] = xmul(lambda[d], ag);
      c[cPenalty + d] = rclamp(xmul(penalty[d], m->gamma), R(1000), R(1e9));
    }
  }

#include "mpr.cuh"

  // Warm-start key of a ground contact: shape and feature (point index).
  static __device__ __forceinline__ int groundKey(int shape, int feature) { return shape << 20 | feature; }

  __device__ __forceinline__ void detectContacts() {
    const int nb = m->nb;
    for (int b = team.lane; b < nb; b += T) I[L.colors + b] = ldg(m->color[b]);
    if (team.lane == 0) I[iColors] = 2;
    const int prevCount = I[iPrevCount];
    // Stage the keys of the previous substep's contacts from the record, one
    // lane per contact, so the lookups below search shared memory.
    {
      const R *prev = rec + kRecHeader + kRecBody * m->nb + kRecJoint * m->nj;
      for (int i = team.lane; i < prevCount; i += T) {
        const R *p = prev + kRecContact * i;
        I[L.prevKeys + i] = p[3] < R(0) ? groundKey(int(p[1]), int(p[2])) : -1;
      }
      team.sync();
    }
    int base = 0;
    for (int first = 0; first < m->ns; first += T) {
      const int s = first + team.lane;
      int feature[4];
      V3<R> world[4];
      int n = s < m->ns ? groundPicks(s, feature, world) : 0;
      int total;
      int offset = team.scan(n, &total);
      if (n > 0) buildGroundPicks(s, n, feature, world, base + offset, prevCount);
      base += total;
    }
    base = base < L.cap ? base : L.cap;
    team.sync();
    if (team.lane == 0) I[iGround] = base;
    if (pairs()) base = detectPairs(base, prevCount);
    if (team.lane == 0) I[iCount] = base;
    team.sync();
    // Per-body masks of the contacts touching each body (list order).
    if (L.cap <= 64) {
      for (int b = team.lane; b < nb; b += T) {
        unsigned long long mask = 0ull;
        for (int c = 0; c < base; ++c) {
          const int meta = cmeta(c);
          if (metaBody(meta) == b || metaOther(meta) == b) mask |= 1ull << c;
        }
        I[L.masks + 2 * b] = int(unsigned(mask));
        I[L.masks + 2 * b + 1] = int(unsigned(mask >> 32));
      }
      team.sync();
    }
  }

  // Colour lists of the dynamic bodies; contacts between equal colours move
  // the second body to a fresh colour (kernel.cuh:717-720).
  __device__ void buildColorLists() {
    if (team.lane == 0) {
      const int nb = m->nb, colorCount = I[iColors];
      int fill = 0;
      for (int c = 0; c < colorCount; ++c) {
        I[L.colorStart + c] = fill;
        for (int b = 0; b < nb; ++b)
          if (I[L.colors + b] == c && ldg(m->mass[b]) > R(0)) I[L.colorList + fill++] = b;
      }
      I[L.colorStart + colorCount] = fill;
    }
    team.sync();
  }

  // ------------------------------------------------------------ joints
  struct JointGeo {
    V3<R> ra, rb, axis, axisB, t1, t2;
    R C[7];
    R angle;
    int a, b, limited;
  };
  // ra, rb, axisA, axisB, tangentA, tangentB, lo, hi of joint j in 128-bit loads.
  __device__ __forceinline__ void loadFrame(int j, R (&f)[20]) const {
    if constexpr (sizeof(R) == 4) {
      const float4 *src = reinterpret_cast<const float4 *>(m->jFrame[j]);
#pragma unroll
      for (int k = 0; k < 5; ++k) {
        float4 v = __ldg(src + k);
        f[4 * k] = v.x; f[4 * k + 1] = v.y; f[4 * k + 2] = v.z; f[4 * k + 3] = v.w;
      }
    } else {
      const double2 *src = reinterpret_cast<const double2 *>(m->jFrame[j]);
#pragma unroll
      for (int k = 0; k < 10; ++k) {
        double2 v = __ldg(src + k);
        f[2 * k] = v.x; f[2 * k + 1] = v.y;
      }
    }
  }
  // Hinge constraint values and world frames (kernel.cuh:725-761).
  __device__ __forceinline__ void evalJoint(int j, JointGeo &e) const {
    const int4 info = __ldg(reinterpret_cast<const int4 *>(m->jInfo[j]));
    e.a = info.x;
    e.b = info.y;
    e.limited = info.z;
    R f[20];
    loadFrame(j, f);
    const SV Ra = rot(e.a), Rb = rot(e.b);
    V3<R> xa = ld3(L.X + 3 * e.a), xb = ld3(L.X + 3 * e.b);
    e.ra = matVec(Ra, V3<R>{f[0], f[1], f[2]});
    e.rb = matVec(Rb, V3<R>{f[3], f[4], f[5]});
    V3<R> d = xa + e.ra - xb - e.rb;
    e.C[0] = d.x; e.C[1] = d.y; e.C[2] = d.z;
    e.axis = matVec(Ra, V3<R>{f[6], f[7], f[8]});
    e.axisB = matVec(Rb, V3<R>{f[9], f[10], f[11]});
    e.t1 = matVec(Ra, V3<R>{f[12], f[13], f[14]});
    e.t2 = cross(e.axis, e.t1);
    e.C[3] = dot(e.t1, e.axisB);
    e.C[4] = dot(e.t2, e.axisB);
    V3<R> u = matVec(Rb, V3<R>{f[15], f[16], f[17]});
    e.angle = fatan2(dot(e.t2, u), dot(e.t1, u));
    e.C[5] = e.angle - f[18];
    e.C[6] = f[19] - e.angle;
  }

  // ------------------------------------------------------------ 6x6 algebra
  // Packed lower triangle: (i, j), j <= i, at i (i + 1) / 2 + j.
  static __device__ __forceinline__ int tri(int i, int j) { return i * (i + 1) / 2 + j; }
  // The three unit-axis rows J_k = (e_k, r x e_k), k = x, y, z, with forces
  // f_k and stiffnesses p_k (hinge anchor rows, ground contacts): the
  // reference's three rank-one stamps (kernel.cuh:164-176) in their order,
  // entry by entry, leaving out the products with a structural zero of
  // r x e_k.
  static __device__ __forceinline__ void stampAxes(R *H, R *g, V3<R> r, R f0, R f1, R f2, R p0, R p1, R p2) {
    // k = x: r x e_x = (0, z, -y).
    g[0] += f0;
    g[4] += r.z * f0; g[5] -= r.y * f0;
    H[tri(0, 0)] += p0;
    H[tri(4, 0)] += p0 * r.z; H[tri(5, 0)] -= p0 * r.y;
    {
      const R py = r.z * p0, pz = r.y * p0;
      H[tri(4, 4)] += py * r.z; H[tri(5, 4)] -= pz * r.z; H[tri(5, 5)] += pz * r.y;
    }
    // k = y: r x e_y = (-z, 0, x).
    g[1] += f1;
    g[3] -= r.z * f1; g[5] += r.x * f1;
    H[tri(1, 1)] += p1;
    H[tri(3, 1)] -= p1 * r.z; H[tri(5, 1)] += p1 * r.x;
    {
      const R px = r.z * p1, pz = r.x * p1;
      H[tri(3, 3)] += px * r.z; H[tri(5, 3)] -= pz * r.z; H[tri(5, 5)] += pz * r.x;
    }
    // k = z: r x e_z = (y, -x, 0).
    g[2] += f2;
    g[3] += r.y * f2; g[4] -= r.x * f2;
    H[tri(2, 2)] += p2;
    H[tri(3, 2)] += p2 * r.y; H[tri(4, 2)] -= p2 * r.x;
    {
      const R px = r.y * p2, py = r.x * p2;
      H[tri(3, 3)] += px * r.y; H[tri(4, 3)] -= py * r.y; H[tri(4, 4)] += py * r.x;
    }
  }
  // Row J = (0, c).
  static __device__ __forceinline__ void stampAngular(R *H, R *g, V3<R> c, R f, R p) {
    g[3] += c.x * f; g[4] += c.y * f; g[5] += c.z * f;
    V3<R> pc = c * p;
    H[tri(3, 3)] += pc.x * c.x;
    H[tri(4, 3)] += pc.y * c.x; H[tri(4, 4)] += pc.y * c.y;
    H[tri(5, 3)] += pc.z * c.x; H[tri(5, 4)] += pc.z * c.y; H[tri(5, 5)] += pc.z * c.z;
  }
  // Dense row J = (e, c).
  static __device__ __forceinline__ void stampDense(R *H, R *g, V3<R> e, V3<R> c, R f, R p) {
    R J[6] = {e.x, e.y, e.z, c.x, c.y, c.z};
#pragma unroll
    for (int i = 0; i < 6; ++i) {
      g[i] += J[i] * f;
      R pj = p * J[i];
#pragma unroll
      for (int k = 0; k <= i; ++k) H[tri(i, k)] += pj * J[k];
    }
  }
  // Diagonal majorizer of the rotational geometric stiffness of force f at
  // lever r: column norms of (r f^T + f r^T) / 2 - (r.f) I (kernel.cuh:283-301).
  static __device__ __forceinline__ void geometric(R *H, V3<R> r, V3<R> f) {
    R rf = dot(r, f);
    R a00 = r.x * f.x - rf, a11 = r.y * f.y - rf, a22 = r.z * f.z - rf;
    R a01 = R(0.5) * (r.x * f.y + f.x * r.y);
    R a02 = R(0.5) * (r.x * f.z + f.x * r.z);
    R a12 = R(0.5) * (r.y * f.z + f.y * r.z);
    H[tri(3, 3)] += fsqrt(a00 * a00 + a01 * a01 + a02 * a02);
    H[tri(4, 4)] += fsqrt(a01 * a01 + a11 * a11 + a12 * a12);
    H[tri(5, 5)] += fsqrt(a02 * a02 + a12 * a12 + a22 * a22);
  }
  // The same majorizer summed over three unit-axis forces f_k e_k at one
  // lever: for f along e_k the column norms are |f_k| times square roots of
  // quadratic forms of r alone.
  static __device__ __forceinline__ void geometricAxes(R *H, V3<R> r, R f0, R f1, R f2) {
    const R x2 = r.x * r.x, y2 = r.y * r.y, z2 = r.z * r.z;
    const R a0 = fabs(f0), a1 = fabs(f1), a2 = fabs(f2);
    H[tri(3, 3)] += a0 * R(0.5) * fsqrt(y2 + z2) + a1 * fsqrt(y2 + R(0.25) * x2) + a2 * fsqrt(z2 + R(0.25) * x2);
    H[tri(4, 4)] += a0 * fsqrt(x2 + R(0.25) * y2) + a1 * R(0.5) * fsqrt(x2 + z2) + a2 * fsqrt(z2 + R(0.25) * y2);
    H[tri(5, 5)] += a0 * fsqrt(x2 + R(0.25) * z2) + a1 * fsqrt(y2 + R(0.25) * z2) + a2 * R(0.5) * fsqrt(x2 + y2);
  }
  // Friction-cone clamped contact force (kernel.cuh:304-315).
  static __device__ __forceinline__ V3<R> coneForce(V3<R> C, SV c) {
    V3<R> f{c[cLambda] + c[cPenalty] * C.x, c[cLambda + 1] + c[cPenalty + 1] * C.y,
            c[cLambda + 2] + c[cPenalty + 2] * C.z};
    f.z = rmin(f.z, R(0));
    R t2 = f.x * f.x + f.y * f.y, bound = -c[cFriction] * f.z;
    if (t2 > bound * bound && t2 > R(0)) {
      R s = bound * frsqrt(t2);
      f.x *= s;
      f.y *= s;
    }
    return f;
  }
  // SO(3) log-Jacobian coefficient (1 - (a/2) cot(a/2)) / a^2 as a function
  // of a^2: its Bernoulli series below 0.5 rad (relative error < 1e-12 there,
  // no square root) and the closed form above, where it has no cancellation.
  static __device__ __forceinline__ R logJacobianCoef(R a2) {
    if (a2 < R(0.25)) {
      return R(1.0 / 12) + a2 * (R(1.0 / 720) + a2 * (R(1.0 / 30240) + a2 * (R(1.0 / 1209600) +
                                                                               a2 * R(1.0 / 47900160))));
    }
    const R a = fsqrt(a2), h = R(0.5) * a;
    R s, c;
    sincosT(h, &s, &c);
    return (R(1) - h * c / s) / a2;
  }
  // Solve H x = -g with a packed Cholesky factorisation (kernel.cuh:177-228);
  // false on a non-positive pivot.
  static __device__ __forceinline__ bool solve(const R *H, const R *g, R *x) {
    R Lf[21], inv[6];
#pragma unroll
    for (int i = 0; i < 6; ++i) {
#pragma unroll
      for (int j = 0; j <= i; ++j) {
        R v = H[tri(i, j)];
#pragma unroll
        for (int k = 0; k < j; ++k) v -= Lf[tri(i, k)] * Lf[tri(j, k)];
        if (i == j) {
          if (!(v > R(0)) || !isfinite(v)) return false;
          R r = frsqrt(v);
          Lf[tri(i, i)] = v * r;
          inv[i] = r;
        } else {
          Lf[tri(i, j)] = v * inv[j];
        }
      }
    }
    R y[6];
#pragma unroll
    for (int i = 0; i < 6; ++i) {
      R v = -g[i];
#pragma unroll
      for (int k = 0; k < i; ++k) v -= Lf[tri(i, k)] * y[k];
      y[i] = v * inv[i];
    }
#pragma unroll
    for (int i = 5; i >= 0; --i) {
      R v = y[i];
#pragma unroll
      for (int k = i + 1; k < 6; ++k) v -= Lf[tri(k, i)] * x[k];
      x[i] = v * inv[i];
    }
    return true;
  }

  // ------------------------------------------------------------ primal
  // A hinge's multipliers and penalties (7 rows) and its dry-friction pair,
  // read once from shared memory and handed to the stamp or the dual update
  // in registers.
  struct Multipliers {
    R lam[7], pen[7], lf, pf;
  };
  __device__ __forceinline__ void loadMultipliers(int j, Multipliers &mu) const {
    const SV lam = S + (L.JL + 7 * j), pen = S + (L.JP + 7 * j);
#pragma unroll
    for (int k = 0; k < 7; ++k) { mu.lam[k] = lam[k]; mu.pen[k] = pen[k]; }
    mu.lf = S[L.JLF + j];
    mu.pf = S[L.JPF + j];
  }
  // Rows of hinge j acting on body bi (kernel.cuh:863-913): anchor rows with
  // their geometric stiffness, axis-orthogonality rows, then limits, PD drive,
  // damping/armature and dry friction summed along the hinge axis.
  __device__ __forceinline__ void stampHinge(int bi, int j, const JointGeo &e, const Multipliers &mu, R *H, R *g, R kp,
                                             R limit) const {
    const R h = sDt, alpha = sAlpha;
    const bool parent = e.a == bi;
    const R s = parent ? R(1) : R(-1);
    const R *lam = mu.lam, *pen = mu.pen;
    const SV c0 = S + (L.JC0 + 7 * j);
    const V3<R> r = parent ? e.ra : e.rb;
    R f3[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      R c = e.C[k] - alpha * c0[k];
      f3[k] = lam[k] + pen[k] * c;
    }
    stampAxes(H, g, r, s * f3[0], s * f3[1], s * f3[2], pen[0], pen[1], pen[2]);
    // Anchor rows: lever (parent ? ra : -rb) under unit-axis forces f_k e_k;
    // the majorizer depends on the lever only through its squares.
    geometricAxes(H, r, f3[0], f3[1], f3[2]);
#pragma unroll
    for (int k = 3; k < 5; ++k) {
      R c = e.C[k] - alpha * c0[k];
      R f = lam[k] + pen[k] * c;
      V3<R> t = k == 3 ? e.t1 : e.t2;
      stampAngular(H, g, cross(t, e.axisB) * s, f, pen[k]);
      geometric(H, parent ? t : e.axisB, (parent ? e.axisB : t) * f);
    }
    // Every remaining row acts along the hinge axis: J = (0, -s axis).
    R stiff = R(0), force = R(0);
    if (e.limited) {
      R c5 = e.C[5] - alpha * rmin(c0[5], R(0));
      R f5 = rmin(lam[5] + pen[5] * c5, R(0));
      if (f5 < R(0)) { stiff += pen[5]; force += f5; }
      R c6 = e.C[6] - alpha * rmin(c0[6], R(0));
      R f6 = rmin(lam[6] + pen[6] * c6, R(0));
      if (f6 < R(0)) { stiff += pen[6]; force -= f6; }
    }
    R drive = kp * wrapAngle(e.angle - S[L.JT + j]) - S[L.JTQ + j];
    R driveStiffness = kp;
    if (limit > R(0)) {
      if (fabs(drive) >= limit) driveStiffness = R(0);
      drive = rclamp(drive, -limit, limit);
    }
    stiff += driveStiffness;
    force += drive;
    const R damping = S[L.JD + j], armature = ldg(m->armature[j]);
    const R delta = wrapAngle(e.angle - S[L.JA0 + j]);
    const R dstiff = damping * ih + armature * ih2;
    if (dstiff > R(0)) {
      stiff += dstiff;
      force += damping * ih * delta + armature * ih2 * (delta - h * S[L.JV0 + j]);
    }
    const R fl = S[L.JFL + j];
    if (fl > R(0)) {
      R trial = mu.lf + mu.pf * delta;
      force += rclamp(trial, -fl, fl);
      if (fabs(trial) < fl) stiff += mu.pf;
    }
    stampAngular(H, g, e.axis * (-s), force, stiff);
  }

  // Rows of contact ci acting on body bi (kernel.cuh:915-927): ground
  // contacts are unit-axis linear rows at lever ra; body pairs are dense rows
  // in the contact basis.  A member function (not a lambda) so that H and g
  // stay in registers.
  __device__ __forceinline__ void stampContact(int bi, int ci, V3<R> x, SV Rb, int nGround, R *H, R *g) const {
    const R alpha = sAlpha;
    const int meta = cmeta(ci);
    const int body = metaBody(meta), other = metaOther(meta);
    const SV c = contact(ci);
    V3<R> local{c[cLocal], c[cLocal + 1], c[cLocal + 2]};
    if (!P || other < 0) {
      V3<R> ra = matVec(Rb, local);
      V3<R> C = x + ra - V3<R>{c[cAnchor], c[cAnchor + 1], c[cAnchor + 2]};
      C.z -= alpha * c[cC0];
      V3<R> f = coneForce(C, c);
      if (f.z < R(0)) {
        stampAxes(H, g, ra, f.x, f.y, f.z, c[cPenalty], c[cPenalty + 1], c[cPenalty + 2]);
        geometric(H, ra, f);
      }
    } else {
      const SV bs = S + (L.CB + 9 * (ci - nGround));
      V3<R> t1{bs[0], bs[1], bs[2]}, t2{bs[3], bs[4], bs[5]}, nn{bs[6], bs[7], bs[8]};
      V3<R> ra = matVec(rot(body), local), rb = matVec(rot(other), V3<R>{c[cAnchor], c[cAnchor + 1], c[cAnchor + 2]});
      V3<R> delta = ld3(L.X + 3 * body) + ra - ld3(L.X + 3 * other) - rb;
      V3<R> C{dot(delta, t1), dot(delta, t2), dot(delta, nn)};
      C.z -= alpha * c[cC0];
      const bool isOther = bi == other;
      const R sign = isOther ? R(-1) : R(1);
      const V3<R> r = isOther ? rb : ra;
      V3<R> f = coneForce(C, c);
      if (f.z < R(0)) {
        V3<R> e0 = t1 * sign, e1 = t2 * sign, e2 = nn * sign;
        stampDense(H, g, e0, cross(r, e0), f.x, c[cPenalty]);
        stampDense(H, g, e1, cross(r, e1), f.y, c[cPenalty + 1]);
        stampDense(H, g, e2, cross(r, e2), f.z, c[cPenalty + 2]);
        geometric(H, r, (t1 * f.x + t2 * f.y + nn * f.z) * sign);
      }
    }
  }

  // Block update of body bi (kernel.cuh:828-936), in two halves:
  // assembleBody forms H and g, applyBody solves and moves the body.
  // With kSplit = 2 the two lanes of a pair (part 0 and 1) take alternate
  // items -- the inertia block, then each hinge, then each contact -- and
  // add their partial H and g with one shuffle per entry; both then solve
  // the same system and part 0 writes the pose.
  // The hinges taken are csrJoint[adjBegin, adjEnd); whole = false (a helper
  // lane of the sweep schedule) leaves out the inertia block and contacts.
  __device__ __forceinline__ void assembleBody(int bi, int adjBegin, int adjEnd, bool whole, R kp, R limit, int part,
                                               R (&H)[21], R (&g)[6]) const {
    const R h = m->dt;
    int item = 0;
    auto mine = [&]() { return kSplit == 1 || (item++ & 1) == part; };
    const R mass = massOf(bi);
#pragma unroll
    for (int i = 0; i < 21; ++i) H[i] = R(0);
#pragma unroll
    for (int i = 0; i < 6; ++i) g[i] = R(0);
    const V3<R> x = ld3(L.X + 3 * bi), xp = ld3(L.XQP + 7 * bi);
    const Q4<R> q = quat(bi), qp = ld4(L.XQP + 7 * bi + 3);
    // Inertia block with the SO(3) log Jacobian and frozen world inertia.
    if (whole && mine()) {
      V3<R> dx = x - xp, th = fqlog(qmul(q, conj(qp)));
      R ml = mass * ih2;
      H[tri(0, 0)] = ml; H[tri(1, 1)] = ml; H[tri(2, 2)] = ml;
      g[0] = ml * dx.x; g[1] = ml * dx.y; g[2] = ml * dx.z;
      R a2 = dot(th, th);
      R coef = logJacobianCoef(a2);
      // rotJ[k] = e_k - theta x e_k / 2 + coef theta x (theta x e_k), as columns.
      R J[3][3];
      R d = R(1) - coef * a2;
      R th3[3] = {th.x, th.y, th.z};
#pragma unroll
      for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int k = 0; k < 3; ++k) J[i][k] = coef * th3[i] * th3[k] + (i == k ? d : R(0));
      // -(theta x e_k) / 2: theta x e_x = (0, tz, -ty), x e_y = (-tz, 0, tx),
      // x e_z = (ty, -tx, 0).
      J[1][0] -= R(0.5) * th.z; J[2][0] += R(0.5) * th.y;
      J[0][1] += R(0.5) * th.z; J[2][1] -= R(0.5) * th.x;
      J[0][2] -= R(0.5) * th.y; J[1][2] += R(0.5) * th.x;
      const SV iw = S + (L.IW + kSIW * bi);   // xx, yy, zz, xy, xz, yz
      R Iw[3][3] = {{iw[0], iw[3], iw[4]}, {iw[3], iw[1], iw[5]}, {iw[4], iw[5], iw[2]}};
      R It[3], N[3][3];
#pragma unroll
      for (int i = 0; i < 3; ++i) {
        It[i] = Iw[i][0] * th.x + Iw[i][1] * th.y + Iw[i][2] * th.z;
#pragma unroll
        for (int l = 0; l < 3; ++l) N[i][l] = Iw[i][0] * J[0][l] + Iw[i][1] * J[1][l] + Iw[i][2] * J[2][l];
      }
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        g[3 + k] = (J[0][k] * It[0] + J[1][k] * It[1] + J[2][k] * It[2]) * ih2;
#pragma unroll
        for (int l = 0; l <= k; ++l)
          H[tri(3 + k, 3 + l)] = (J[0][k] * N[0][l] + J[1][k] * N[1][l] + J[2][k] * N[2][l]) * ih2;
      }
    }
    // Hinges touching bi, in CSR order.  One inlined copy of the hinge rows:
    // the Gauss-Seidel loop is instruction-fetch bound, so its code is kept
    // small rather than unrolled over hinge pairs.
    for (int adj = adjBegin; adj < adjEnd; ++adj) {
      if (!mine()) continue;
      const int j = ldg(m->csrJoint[adj]);
      JointGeo e;
      evalJoint(j, e);
      Multipliers mu;
      loadMultipliers(j, mu);
      stampHinge(bi, j, e, mu, H, g, kp, limit);
    }
    // Contacts touching bi, in list order.
    const int nGround = I[iGround];
    const SV Rb = rot(bi);
    // One loop (one inlined copy of the contact rows) over the contacts that
    // touch bi, in list order: from the per-body bit mask when the list fits
    // 64 entries, else by scanning the list.
    const bool useMask = L.cap <= 64;
    unsigned long long mask = useMask && whole ? unsigned(I[L.masks + 2 * bi]) |
                                                     (unsigned long long)unsigned(I[L.masks + 2 * bi + 1]) << 32
                                               : 0ull;
    const int count = useMask || !whole ? 0 : I[iCount];
    int scan = 0;
    for (;;) {
      int ci = -1;
      if (useMask) {
        if (!mask) break;
        ci = __ffsll((long long)mask) - 1;
        mask &= mask - 1;
      } else {
        while (scan < count) {
          const int meta = cmeta(scan);
          if (metaBody(meta) == bi || metaOther(meta) == bi) break;
          ++scan;
        }
        if (scan >= count) break;
        ci = scan++;
      }
      if (mine()) stampContact(bi, ci, x, Rb, nGround, H, g);
    }
    if constexpr (kSplit == 2) {
      const unsigned pair = 3u << ((threadIdx.x & 31) & ~1);
#pragma unroll
      for (int i = 0; i < 21; ++i) H[i] += __shfl_xor_sync(pair, H[i], 1);
#pragma unroll
      for (int i = 0; i < 6; ++i) g[i] += __shfl_xor_sync(pair, g[i], 1);
    }
  }

  // Solve H st = -g, clamp the step (0.1 m, 0.25 rad) and move body bi;
  // returns the square of the applied step length (kernel.cuh:928-936).  An
  // unclamped step (the usual case) needs no square root or reciprocal.
  __device__ __forceinline__ R applyBody(int bi, const R (&H)[21], const R (&g)[6], int part) {
    const V3<R> x = ld3(L.X + 3 * bi);
    const Q4<R> q = quat(bi);
    R st[6];
    if (!solve(H, g, st)) {
#pragma unroll
      for (int i = 0; i < 6; ++i) st[i] = R(NAN);
    }
    V3<R> tx{st[0], st[1], st[2]}, rx{st[3], st[4], st[5]};
    const R nt2 = dot(tx, tx), nr2 = dot(rx, rx);
    R scale = R(1);
    if (nt2 > R(0.01) || nr2 > R(0.0625)) {
      const R nt = fsqrt(nt2), nr = fsqrt(nr2);
      scale = rmin(R(1), rmin(R(.1) * frcp(rmax(nt, R(1e-30))), R(.25) * frcp(rmax(nr, R(1e-30)))));
    }
    if (part == 0) setPose(bi, x + tx * scale, fnormalized(qmul(fqexpRaw(rx * scale), q)));
    return rmax(nt2, nr2) * scale * scale;
  }

  // Dual update of hinge j (kernel.cuh:991-1028): multipliers, penalty ramps,
  // dry friction; folds the constraint error into *error.
  __device__ __forceinline__ void dualHinge(int j, const JointGeo &e, R &error, Multipliers &mu) const {
    const R alpha = sAlpha;
    const SV lam = S + (L.JL + 7 * j), pen = S + (L.JP + 7 * j), c0 = S + (L.JC0 + 7 * j);
    const int rows = e.limited ? 7 : 5;
#pragma unroll
    for (int k = 0; k < 7; ++k) {
      if (k >= rows) break;
      R c = e.C[k] - alpha * (k < 5 ? c0[k] : rmin(c0[k], R(0)));
      R f = mu.lam[k] + mu.pen[k] * c;
      mu.lam[k] = k >= 5 ? rmin(f, R(0)) : f;
      lam[k] = mu.lam[k];
      if (k < 5 || f < R(0)) {
        mu.pen[k] = rmin(mu.pen[k] + (k < 3 ? sBetaL : sBetaA) * fabs(c), k < 3 ? R(1e9) : R(1e7));
        pen[k] = mu.pen[k];
      }
      error = rmax(error, k < 5 ? R(fabs(c)) : rmax(R(0), -c));
    }
    const R fl = S[L.JFL + j];
    if (fl > R(0)) {
      R delta = wrapAngle(e.angle - S[L.JA0 + j]);
      R trial = mu.lf + mu.pf * delta;
      R lf = rclamp(trial, -fl, fl);
      R pf = mu.pf;
      if (fabs(trial) < fl) pf = rmin(pf + sBetaA * R(fabs(delta)), R(1e7));
      mu.lf = lf;
      mu.pf = pf;
      S[L.JLF + j] = lf;
      S[L.JPF + j] = pf;
      R residual = lf + pf * delta;
      error = rmax(error, R(fabs(lf - rclamp(residual, -fl, fl))) * frcp(pf));
    }
  }

  // Contact gap C in the contact basis, C.z shifted by -alpha c0 (kernel.cuh:805-827).
  __device__ __forceinline__ V3<R> contactGap(int ci, int nGround) const {
    const SV c = contact(ci);
    const int meta = cmeta(ci);
    const int body = metaBody(meta), other = metaOther(meta);
    V3<R> local{c[cLocal], c[cLocal + 1], c[cLocal + 2]};
    V3<R> ra = matVec(rot(body), local);
    V3<R> C;
    if (!P || other < 0) {
      C = ld3(L.X + 3 * body) + ra - V3<R>{c[cAnchor], c[cAnchor + 1], c[cAnchor + 2]};
    } else {
      const SV bs = S + (L.CB + 9 * (ci - nGround));
      V3<R> rb = matVec(rot(other), V3<R>{c[cAnchor], c[cAnchor + 1], c[cAnchor + 2]});
      V3<R> delta = ld3(L.X + 3 * body) + ra - ld3(L.X + 3 * other) - rb;
      C = {dot(delta, V3<R>{bs[0], bs[1], bs[2]}), dot(delta, V3<R>{bs[3], bs[4], bs[5]}),
           dot(delta, V3<R>{bs[6], bs[7], bs[8]})};
    }
    C.z -= sAlpha * c[cC0];
    return C;
  }

  // Start-of-substep hinge values, angle and axis rate (kernel.cuh:951-964).
  __device__ __forceinline__ void setJointStart(int j, const JointGeo &e) {
#pragma unroll
    for (int k = 0; k < 7; ++k) S[L.JC0 + 7 * j + k] = e.C[k];
    S[L.JA0 + j] = e.angle;
    S[L.JV0 + j] = dot(omega(e.b) - omega(e.a), e.axis);
  }

  // ------------------------------------------------------------ substep
  struct Diag {
    R jointError, axisError, penetration;
    int contacts, iterations;
    bool converged;
  };

  // cached: the previous substep of this call ended with the diagnostics
  // pass, which left this substep's hinge values, angles and axis rates in
  // JC0, JA0 and JV0 (the poses and velocities have not moved since).
  __device__ __forceinline__ bool step(Diag &diag, R kp, R limit, bool cached) {
    const R h = m->dt, alpha = m->alpha, gamma = m->gamma;
    diag = {R(0), R(0), R(0), 0, 0, false};
    detectContacts();
    if (pairs()) buildColorLists();
    if (I[iFailed]) {
      storeContacts();
      return false;
    }
    const int nb = m->nb, nj = m->nj;
    const R ag = alpha * gamma;
    // Joint warm start (kernel.cuh:951-964), one lane per joint.
    for (int j = team.lane; j < nj; j += T) {
      if (!cached) {
        JointGeo e;
        evalJoint(j, e);
        setJointStart(j, e);
      }
      S[L.JLF + j] *= ag;
      S[L.JPF + j] = rclamp(S[L.JPF + j] * gamma, R(1), R(1e7));
#pragma unroll
      for (int k = 0; k < 7; ++k) {
        S[L.JL + 7 * j + k] *= ag;
        R p = S[L.JP + 7 * j + k] * gamma;
        S[L.JP + 7 * j + k] = k < 3 ? rclamp(p, R(1000), R(1e9)) : rclamp(p, R(1), R(1e7));
      }
    }
    team.sync();
    // Predictor (kernel.cuh:965-976), one lane per body.  The predicted pose
    // takes over the velocity slots of the body.  x0 and q0 wait for velocity
    // recovery (the same lane, the same body) in registers when the model has
    // no body pairs; the pair instantiation, short of registers, parks them in
    // the body's pose slots of the record, which nothing reads before store()
    // rewrites them at the end of the call.
    V3<R> x0r[P ? 1 : kPerLane];
    Q4<R> q0r[P ? 1 : kPerLane];
#pragma unroll
    for (int k = 0; k < kPerLane; ++k) {
      const int b = team.lane + k * T;
      if (b >= nb) continue;
      const V3<R> x = ld3(L.X + 3 * b);
      const Q4<R> q = quat(b);
      if constexpr (P) {
        R *r0 = rec + kRecHeader + kRecBody * b;
        r0[0] = x.x; r0[1] = x.y; r0[2] = x.z; r0[3] = q.w; r0[4] = q.x; r0[5] = q.y; r0[6] = q.z;
      } else {
        x0r[k] = x; q0r[k] = q;
      }
      const R mass = massOf(b);
      if (mass == R(0)) continue;
      V3<R> in = inertiaOf(b);
      // World inertia R diag(I) R^T at q0 (kept for the whole substep).
      const SV Rm = rot(b);
      V3<R> ex{Rm[0], Rm[3], Rm[6]}, ey{Rm[1], Rm[4], Rm[7]}, ez{Rm[2], Rm[5], Rm[8]};
      SV iw = S + (L.IW + kSIW * b);
      iw[0] = in.x * ex.x * ex.x + in.y * ey.x * ey.x + in.z * ez.x * ez.x;
      iw[1] = in.x * ex.y * ex.y + in.y * ey.y * ey.y + in.z * ez.y * ez.y;
      iw[2] = in.x * ex.z * ex.z + in.y * ey.z * ey.z + in.z * ez.z * ez.z;
      iw[3] = in.x * ex.x * ex.y + in.y * ey.x * ey.y + in.z * ez.x * ez.y;
      iw[4] = in.x * ex.x * ex.z + in.y * ey.x * ey.z + in.z * ez.x * ez.z;
      iw[5] = in.x * ex.y * ex.z + in.y * ey.y * ey.z + in.z * ez.y * ez.z;
      V3<R> v = vel(b), w = omega(b);
      V3<R> grav{m->gravity[0], m->gravity[1], m->gravity[2]};
      V3<R> xp = x + v * h + (grav + bodyForce(b) * (R(1) / mass)) * (h * h);
      // Gyroscopic predictor: w + h I^-1 (-(w x I w)), body frame.
      V3<R> wl{ex.x * w.x + ex.y * w.y + ex.z * w.z, ey.x * w.x + ey.y * w.y + ey.z * w.z,
               ez.x * w.x + ez.y * w.y + ez.z * w.z};
      V3<R> Iwl{in.x * wl.x, in.y * wl.y, in.z * wl.z};
      V3<R> tl = -cross(wl, Iwl);
      V3<R> wp = w + matVec(Rm, V3<R>{tl.x / in.x, tl.y / in.y, tl.z / in.z}) * h;
      Q4<R> qp = qmul(fqexp(wp * h), q);
      SV xqp = S + (L.XQP + 7 * b);
      xqp[0] = xp.x; xqp[1] = xp.y; xqp[2] = xp.z;
      xqp[3] = qp.w; xqp[4] = qp.x; xqp[5] = qp.y; xqp[6] = qp.z;
      setPose(b, xp, qp);
    }
    team.sync();
    const int colorCount = pairs() ? I[iColors] : 2;
    const R tol = m->tolerance;
    const int iterations = m->iterations;
    for (int it = 0; it < iterations; ++it) {
      R maxUpdate = R(0);
      for (int color = 0; color < colorCount; ++color) {
        int begin, end;
        if (pairs()) {
          begin = I[L.colorStart + color];
          end = I[L.colorStart + color + 1];
        } else {
          begin = ldg(m->colorStart[color]);
          end = ldg(m->colorStart[color + 1]);
        }
        // Scheduled colours (scheduleSweep) give each lane at most one role.
        const bool scheduled = color < 2 && m->sweepScheduled;
        int slot = begin + team.lane / kSplit;
        do {
          int bi = -1, adjBegin = 0, adjEnd = 0, role = -1;
          if (scheduled) {
            const int4 sc = __ldg(reinterpret_cast<const int4 *>(m->sweep[color][team.lane]));
            bi = sc.x;
            adjBegin = sc.y;
            adjEnd = sc.z;
            role = sc.w;
          } else if (slot < end) {
            bi = pairs() ? I[L.colorList + slot] : ldg(m->colorBody[slot]);
            adjBegin = ldg(m->csrOffset[bi]);
            adjEnd = ldg(m->csrOffset[bi + 1]);
          }
          const bool have = bi >= 0, owner = role < 32;
          R H[21], g[6];
          if (have) assembleBody(bi, adjBegin, adjEnd, owner, kp, limit, team.lane % kSplit, H, g);
          if (scheduled && m->sweepHelpers[color]) {
            // An owner adds its helper's partial H and g (team-wide shuffles).
            const int src = role >= 0 && role < 32 ? role : team.lane;
#pragma unroll
            for (int i = 0; i < 21; ++i) {
              const R v = __shfl_sync(team.mask, H[i], src, T);
              if (src != team.lane) H[i] += v;
            }
#pragma unroll
            for (int i = 0; i < 6; ++i) {
              const R v = __shfl_sync(team.mask, g[i], src, T);
              if (src != team.lane) g[i] += v;
            }
          }
          if (have && owner) maxUpdate = rmax(maxUpdate, applyBody(bi, H, g, team.lane % kSplit));
          slot += T / kSplit;
        } while (!scheduled && slot < end);
        team.sync();
      }
      maxUpdate = team.max(maxUpdate);
      R error = R(0);
      // Joint multipliers, penalties and dry friction (kernel.cuh:991-1028).
      for (int j = team.lane; j < nj; j += T) {
        JointGeo e;
        evalJoint(j, e);
        Multipliers mu;
        loadMultipliers(j, mu);
        dualHinge(j, e, error, mu);
      }
      // Contact multipliers, stick flags and penalties (kernel.cuh:1029-1052).
      const int n = I[iCount], nGround = I[iGround];
      for (int ci = team.lane; ci < n; ci += T) {
        const SV c = contact(ci);
        const V3<R> C = contactGap(ci, nGround);
        V3<R> f = coneForce(C, c);
        R tx = c[cLambda] + c[cPenalty] * C.x, ty = c[cLambda + 1] + c[cPenalty + 1] * C.y;
        R trial = fsqrt(tx * tx + ty * ty);
        const R mu = c[cFriction];
        const bool cone = trial <= -mu * f.z;
        const bool stick = cone && C.x * C.x + C.y * C.y < R(1e-10);
        const int meta = cmeta(ci);
        cmeta(ci) = (meta & ~(1 << 11)) | (stick ? 1 << 11 : 0);
        R Ck[3] = {C.x, C.y, C.z}, fk[3] = {f.x, f.y, f.z};
#pragma unroll
        for (int k = 0; k < 3; ++k) {
          c[cLambda + k] = fk[k];
          if (f.z < R(0) && (k == 2 || cone))
            c[cPenalty + k] = rmin(c[cPenalty + k] + sBetaL * R(fabs(Ck[k])), R(1e9));
        }
        error = rmax(error, rmax(R(0), -C.z));
      }
      error = team.max(error);
      team.sync();
      diag.iterations = it + 1;
      // maxUpdate holds squared step lengths.
      diag.converged = maxUpdate < tol * tol && error < tol;
      if (diag.converged) break;
    }
    // Velocity recovery (kernel.cuh:1064-1073); the velocities return to the
    // XQP slots.
    bool bad = false;
#pragma unroll
    for (int k = 0; k < kPerLane; ++k) {
      const int b = team.lane + k * T;
      if (b >= nb || !(ldg(m->mass[b]) > R(0))) continue;
      V3<R> x = ld3(L.X + 3 * b);
      V3<R> x0;
      Q4<R> q0;
      if constexpr (P) {
        const R *r0 = rec + kRecHeader + kRecBody * b;
        x0 = {r0[0], r0[1], r0[2]};
        q0 = {r0[3], r0[4], r0[5], r0[6]};
      } else {
        x0 = x0r[k];
        q0 = q0r[k];
      }
      V3<R> v = (x - x0) * ih;
      V3<R> w = fqlog(qmul(quat(b), conj(q0))) * ih;
      SV vw = S + (L.XQP + 7 * b);
      vw[0] = v.x; vw[1] = v.y; vw[2] = v.z; vw[3] = w.x; vw[4] = w.y; vw[5] = w.z;
      if (!isfinite(dot(x, x) + dot(v, v) + dot(w, w))) bad = true;
    }
    if (team.any(bad)) {
      if (team.lane == 0) I[iFailed] = 1;
      team.sync();
      storeContacts();
      return false;
    }
    // Diagnostics (kernel.cuh:1074-1093).
    R je = R(0), ae = R(0), pe = R(0);
    for (int j = team.lane; j < nj; j += T) {
      JointGeo e;
      evalJoint(j, e);
      setJointStart(j, e);   // the next substep's start values
      je = rmax(je, rmax(R(fabs(e.C[0])), rmax(R(fabs(e.C[1])), R(fabs(e.C[2])))));
      ae = rmax(ae, rmax(R(fabs(e.C[3])), R(fabs(e.C[4]))));
    }
    const int n = I[iCount], nGround = I[iGround];
    for (int ci = team.lane; ci < n; ci += T) {
      V3<R> C = contactGap(ci, nGround);
      pe = rmax(pe, rmax(R(0), -(C.z + alpha * contact(ci)[cC0])));
    }
    diag.jointError = team.max(je);
    diag.axisError = team.max(ae);
    diag.penetration = team.max(pe);
    diag.contacts = n;
    team.sync();
    storeContacts();
    return true;
  }

  // BasicState::advance (kernel.cuh:421-443).
  __device__ __forceinline__ void advance(int substeps, R kp, R limit, Diag &summary) {
    summary = {R(0), R(0), R(0), 0, 0, true};
    const R h = m->dt;
    if (!(h > R(0)) || m->iterations < 1) {
      if (team.lane == 0) I[iFailed] = 1;
      team.sync();
      return;
    }
    for (int k = 0; k < substeps; ++k) {
      Diag d;
      bool ok = step(d, kp, limit, k > 0);
      team.sync();
      if (!ok || I[iFailed]) break;
      summary.jointError = rmax(summary.jointError, d.jointError);
      summary.axisError = rmax(summary.axisError, d.axisError);
      summary.penetration = rmax(summary.penetration, d.penetration);
      summary.contacts = summary.contacts > d.contacts ? summary.contacts : d.contacts;
      summary.converged = summary.converged && d.converged;
      summary.iterations += d.iterations;
      // The next substep reads the contacts just stored as its warm-start cache.
      if (team.lane == 0) I[iPrevCount] = I[iCount];
      team.sync();
    }
  }
};

// One launch advances every environment: target/forces (step) or motor/forces
// (step_motor), then `substeps` physics steps with all state on chip.
template <class R, int T, bool P>
__global__ void __launch_bounds__(32, T >= 16 ? 14 : 1) advanceKernel(const DevModel<R> *__restrict__ model,
                                                    const R *__restrict__ points, R *records,
                                                    int recordStride, int count, const __grid_constant__ Layout L,
                                                    StepArgs args) {
  extern __shared__ __align__(16) unsigned char smemRaw[];
  constexpr int teams = 32 / T;
  const int team = threadIdx.x / T;
  const int env = blockIdx.x * teams + team;
  if (env >= count) return;
  // Teams are interleaved word by word: team t owns words t, t + teams, ...
  R *teamBase = reinterpret_cast<R *>(smemRaw) + team;
  R *rec = records + size_t(env) * recordStride;
  Solver<R, T, P> s(model, points, teamBase, rec, L);
  if (args.mass) s.envMass = static_cast<const R *>(args.mass) + size_t(env) * model->nb;
  if (args.inertia) s.envInertia = static_cast<const R *>(args.inertia) + size_t(env) * model->nb * 3;
  if (args.friction) s.envFriction = static_cast<const R *>(args.friction) + size_t(env) * model->ns;
  const typename Solver<R, T, P>::SV S = s.S;
  const int nj = model->nj;
  const int lane = s.team.lane;
  const R *forces = static_cast<const R *>(args.forces) + 3 * size_t(env);
  R kp, limit;
  int failed = int(rec[0]);
  if (args.motor) {
    // BasicState::setMotor (kernel.cuh:448-466): kp and the PD cap are zero,
    // the three channels replace torque, dry friction and damping.
    const R *motor = static_cast<const R *>(args.motor) + size_t(env) * nj * 3;
    kp = R(0);
    limit = R(0);
    bool bad = false;
    for (int j = lane; j < nj; j += T) {
      R t = motor[3 * j], fr = motor[3 * j + 1], dm = motor[3 * j + 2];
      if (!isfinite(t) || !isfinite(fr) || !isfinite(dm) || fr < R(0) || dm < R(0)) bad = true;
    }
    for (int k = lane; k < 3; k += T)
      if (!isfinite(forces[k])) bad = true;
    failed |= s.team.any(bad) ? 1 : 0;
    s.load();
    s.team.sync();
    for (int j = lane; j < nj; j += T) {
      S[L.JTQ + j] = motor[3 * j];
      S[L.JFL + j] = motor[3 * j + 1];
      S[L.JD + j] = motor[3 * j + 2];
    }
    if (lane == 0) {
      S[L.F1] = forces[0]; S[L.F1 + 1] = forces[1]; S[L.F1 + 2] = forces[2];
      s.I[iFailed] = failed;
    }
    s.team.sync();
    typename Solver<R, T, P>::Diag d{R(0), R(0), R(0), 0, 0, true};
    bool ran = !failed;
    if (ran) s.advance(1, kp, limit, d);
    s.team.sync();
    s.store(kp, limit);
    if (ran) s.storeHeader(d.jointError, d.penetration, d.contacts, d.converged, d.axisError, d.iterations);
    else if (lane == 0) rec[0] = R(1);
    return;
  }
  // extension.cu:87-110: validate, then set the PD targets and gains.
  const R *target = static_cast<const R *>(args.target) + size_t(env) * nj;
  bool bad = false;
  for (int j = lane; j < nj; j += T)
    if (!isfinite(target[j])) bad = true;
  for (int k = lane; k < 3; k += T)
    if (!isfinite(forces[k])) bad = true;
  if (s.team.any(bad)) failed = 1;
  if (failed) {
    if (lane == 0) rec[0] = R(1);
    return;
  }
  kp = R(args.kp);
  limit = R(args.limit);
  s.load();
  s.team.sync();
  for (int j = lane; j < nj; j += T) {
    S[L.JT + j] = target[j];
    S[L.JTQ + j] = ldg(model->torque[j]);
    S[L.JFL + j] = ldg(model->frictionloss[j]);
    S[L.JD + j] = ldg(model->damping[j]);
  }
  if (lane == 0) {
    S[L.F1] = forces[0]; S[L.F1 + 1] = forces[1]; S[L.F1 + 2] = forces[2];
    s.I[iFailed] = 0;
  }
  s.team.sync();
  typename Solver<R, T, P>::Diag d;
  s.advance(args.substeps, kp, limit, d);
  s.team.sync();
  s.store(kp, limit);
  s.storeHeader(d.jointError, d.penetration, d.contacts, d.converged, d.axisError, d.iterations);
}

}  // namespace duckb200
