// Host side: DUCK_MODEL text loader and conversion to the flat device model.
//
// Loader semantics follow the reference's duck::Solver::load
// (src/solver.cpp:67-174): the same fields, validation rules and messages,
// quaternions normalised and unit vectors computed in double.  Conversion
// follows duck_native::convert (src/cuda/model.hpp:237-360): capacity and
// topology checks, the two-colouring of the hinge tree, the body->joint CSR
// and the convex point pool.  The result is a plain struct the kernels read
// through the read-only data path, plus a few derived tables the B200 kernels
// use (per-colour body lists, team size, on-chip contact capacity).
#pragma once
#include <algorithm>
#include <cmath>
#include <fstream>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <vector>

namespace duckb200 {

// The reference caps body-collision pairs at 32 (solver.cpp:151-152,
// model.hpp:26-29); kReferencePairs keeps that limit by default.  Batches
// created with a larger pair limit (up to kMaxPairs) accept models with more
// pairs -- an extension beyond the reference.
constexpr int kMaxBodies = 32, kMaxJoints = 32, kMaxShapes = 32, kMaxPairs = 128, kReferencePairs = 32;

template <class R> struct DevModel {
  int nb, nj, ns, np;
  int bound;         // contact bound of the portable record: pairs + 4 per ground shape
  int groundCap;     // on-chip ground contact capacity: sum of min(4, points) per ground shape
  int colorMax;      // largest number of dynamic bodies sharing one hinge colour
  // Sweep schedule of the two model colours for the batch's team width, set
  // by scheduleSweep (1 lane per body only): lane l of colour c handles body
  // sweep[c][l][0] (-1: idle) and its hinges csrJoint[sweep[c][l][1] ..
  // sweep[c][l][2]).  sweep[c][l][3] is -1 for a lane that owns its body
  // alone, the helper's lane for an owner with a helper, and 32 + the owner's
  // lane for a helper, which stamps only its hinges and hands its partial H
  // and g to the owner.  sweepHelpers[c] = 1 when colour c has a helper.
  int sweepScheduled, sweepHelpers[2];
  alignas(16) int sweep[2][32][4];
  int ground, iterations;
  R dt, alpha, gamma, betaLinear, betaAngular, tolerance;
  R gravity[3];
  // bodies
  R mass[kMaxBodies], inertia[kMaxBodies][3];
  R x[kMaxBodies][3], q[kMaxBodies][4], v[kMaxBodies][3], w[kMaxBodies][3];
  int color[kMaxBodies];
  int csrOffset[kMaxBodies + 1], csrJoint[2 * kMaxJoints];
  int colorStart[3], colorBody[kMaxBodies];   // dynamic bodies of model colours 0 and 1
  // joints
  int ja[kMaxJoints], jb[kMaxJoints], limited[kMaxJoints];
  R ra[kMaxJoints][3], rb[kMaxJoints][3], axisA[kMaxJoints][3], axisB[kMaxJoints][3];
  R tangentA[kMaxJoints][3], tangentB[kMaxJoints][3];
  R lo[kMaxJoints], hi[kMaxJoints], damping[kMaxJoints], armature[kMaxJoints];
  R frictionloss[kMaxJoints], torque[kMaxJoints], kp[kMaxJoints], target[kMaxJoints];
  R maxTorque[kMaxJoints];
  // Hot copies for the step kernel, laid out for 128-bit loads: per joint
  // (a, b, limited, 0) and ra, rb, axisA, axisB, tangentA, tangentB, lo, hi.
  alignas(16) int jInfo[kMaxJoints][4];
  alignas(16) R jFrame[kMaxJoints][20];
  // shapes
  int sBody[kMaxShapes], sType[kMaxShapes], sOffset[kMaxShapes], sCount[kMaxShapes];
  int sGround[kMaxShapes];
  R sCenter[kMaxShapes][3], sSize[kMaxShapes][3], sInterior[kMaxShapes][3], sQ[kMaxShapes][4];
  R sFriction[kMaxShapes], sRadius[kMaxShapes];
  // collision pairs
  int pA[kMaxPairs], pB[kMaxPairs];
  R pFriction[kMaxPairs];
};

// Lanes of a team sweep one colour at a time, one body per lane, and a warp
// runs as long as its busiest lane: the body with the most hinges sets the
// pace.  Where a colour has fewer bodies than the team has lanes, the spare
// lanes help the bodies with the most hinges, taking the second half of
// their hinge list, as long as that lowers the colour's largest hinge count.
// Only models whose colours never change (no body-collision pairs) and teams
// of one lane per body (T <= 8) are scheduled.
template <class R> void scheduleSweep(DevModel<R> &d, int T) {
  d.sweepScheduled = 0;
  d.sweepHelpers[0] = d.sweepHelpers[1] = 0;
  if (d.np != 0 || T > 8) return;
  for (int c = 0; c < 2; ++c)
    if (d.colorStart[c + 1] - d.colorStart[c] > T) return;
  for (int c = 0; c < 2; ++c) {
    int owner[32], begin[32], end[32], role[32];
    const int n = d.colorStart[c + 1] - d.colorStart[c];
    for (int l = 0; l < 32; ++l) { owner[l] = -1; begin[l] = end[l] = 0; role[l] = -1; }
    for (int l = 0; l < n; ++l) {
      const int b = d.colorBody[d.colorStart[c] + l];
      owner[l] = b;
      begin[l] = d.csrOffset[b];
      end[l] = d.csrOffset[b + 1];
    }
    int spare = T - n, next = n;
    for (;;) {
      int most = 0, count = 0;
      for (int l = 0; l < next; ++l) most = std::max(most, end[l] - begin[l]);
      for (int l = 0; l < next; ++l) count += end[l] - begin[l] == most;
      if (most < 2 || count > spare) break;
      for (int l = 0, hi = next; l < hi; ++l) {
        if (end[l] - begin[l] != most || role[l] >= 32) continue;
        if (role[l] >= 0) { spare = 0; break; }   // one helper per owner
        const int h = next++;
        const int keep = (most + 1) / 2;
        owner[h] = owner[l];
        begin[h] = begin[l] + keep;
        end[h] = end[l];
        end[l] = begin[l] + keep;
        role[l] = h;
        role[h] = 32 + l;
        --spare;
        d.sweepHelpers[c] = 1;
      }
      if (spare <= 0) break;
    }
    for (int l = 0; l < 32; ++l) {
      d.sweep[c][l][0] = owner[l];
      d.sweep[c][l][1] = begin[l];
      d.sweep[c][l][2] = end[l];
      d.sweep[c][l][3] = role[l];
    }
  }
  d.sweepScheduled = 1;
}

struct DVec { double x = 0, y = 0, z = 0; };
struct DQuat { double w = 1, x = 0, y = 0, z = 0; };

inline DVec dcross(DVec a, DVec b) {
  return {a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x};
}
inline double ddot(DVec a, DVec b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
inline DVec dadd(DVec a, DVec b) { return {a.x + b.x, a.y + b.y, a.z + b.z}; }
inline DVec dscale(DVec a, double s) { return {a.x * s, a.y * s, a.z * s}; }
inline DVec drotate(DQuat q, DVec v) {
  DVec u{q.x, q.y, q.z};
  return dadd(v, dscale(dcross(u, dadd(dcross(u, v), dscale(v, q.w))), 2));
}

struct ParsedModel {
  struct Body { std::string name; double mass = 0; DVec inertia, x, v, w; DQuat q; };
  struct Joint {
    std::string name;
    int a = 0, b = 0;
    DVec ra, rb, axisA, axisB, tangentA, tangentB;
    bool limited = false;
    double lo = 0, hi = 0, damping = 0, armature = 0, frictionloss = 0, torque = 0, kp = 0,
           target = 0, maxTorque = 0;
  };
  struct Shape {
    int body = 0, type = 0;
    DVec center, size;
    DQuat q;
    double friction = 0.8, boundingRadius = 0;
    std::vector<DVec> localPoints;
    bool ground = true;
  };
  struct Pair { int a = 0, b = 0; double friction = 0; };
  DVec gravity{0, 0, -9.81};
  bool ground = false;
  std::vector<Body> bodies;
  std::vector<Joint> joints;
  std::vector<Shape> shapes;
  std::vector<Pair> pairs;
};

inline ParsedModel parseDuck(const std::string &path, int maxPairs = kReferencePairs) {
  std::ifstream in(path);
  if (!in) throw std::runtime_error("Cannot read model: " + path);
  auto unitOf = [](DVec a) {
    double n = std::sqrt(ddot(a, a));
    if (n < 1e-15) throw std::runtime_error("Zero direction");
    return dscale(a, 1 / n);
  };
  auto readV = [&] { DVec v; in >> v.x >> v.y >> v.z; return v; };
  auto readQ = [&] {
    DQuat q;
    in >> q.w >> q.x >> q.y >> q.z;
    double n = std::sqrt(q.w * q.w + q.x * q.x + q.y * q.y + q.z * q.z);
    if (n < 1e-15) throw std::runtime_error("Zero quaternion");
    return DQuat{q.w / n, q.x / n, q.y / n, q.z / n};
  };
  ParsedModel m;
  std::string header;
  int version = -1, nb = -1, nj = -1, ns = -1;
  in >> header >> version >> nb >> nj >> ns;
  if (header != "DUCK_MODEL" || (version != 1 && version != 2) || nb < 1 || nb > 10000 ||
      nj < 0 || ns < 0)
    throw std::runtime_error("Invalid model header");
  m.gravity = readV();
  in >> m.ground;
  m.bodies.resize(nb);
  m.joints.resize(nj);
  m.shapes.resize(ns);
  for (auto &b : m.bodies) {
    in >> b.name >> b.mass;
    b.inertia = readV(); b.x = readV(); b.q = readQ(); b.v = readV(); b.w = readV();
    if (b.mass < 0 || (b.mass > 0 && (b.inertia.x <= 0 || b.inertia.y <= 0 || b.inertia.z <= 0)))
      throw std::runtime_error("Invalid mass/inertia");
  }
  for (auto &j : m.joints) {
    in >> j.name >> j.a >> j.b;
    j.ra = readV(); j.rb = readV();
    j.axisA = unitOf(readV()); j.axisB = unitOf(readV());
    j.tangentA = unitOf(readV()); j.tangentB = unitOf(readV());
    in >> j.limited >> j.lo >> j.hi >> j.damping >> j.armature >> j.frictionloss >> j.torque >>
        j.kp >> j.target >> j.maxTorque;
    if (j.a < 0 || j.b < 0 || j.a >= nb || j.b >= nb || j.a == j.b || j.damping < 0 ||
        j.armature < 0 || j.frictionloss < 0)
      throw std::runtime_error("Invalid joint");
  }
  for (auto &s : m.shapes) {
    int n = -1;
    in >> s.body >> s.type;
    s.center = readV(); s.q = readQ(); s.size = readV();
    in >> s.friction >> n;
    if (s.body < 0 || s.body >= nb || s.type < 0 || s.type > 3 || n < 0 || n > 1000000 ||
        s.friction < 0)
      throw std::runtime_error("Invalid collision shape");
    std::vector<DVec> vertices;
    for (int k = 0; k < n; ++k) vertices.push_back(readV());
    if (version == 2) in >> s.ground;
    if (s.type == 3 && n < 4) throw std::runtime_error("Convex mesh needs at least four vertices");
    if (s.type == 1) {
      for (int i = 0; i < 8; ++i)
        s.localPoints.push_back(dadd(s.center, drotate(s.q, DVec{(i & 1 ? 1 : -1) * s.size.x,
                                                                 (i & 2 ? 1 : -1) * s.size.y,
                                                                 (i & 4 ? 1 : -1) * s.size.z})));
    } else if (s.type == 3) {
      for (auto v : vertices) s.localPoints.push_back(dadd(s.center, drotate(s.q, v)));
    }
    for (auto p : s.localPoints) s.boundingRadius = std::max(s.boundingRadius, std::sqrt(ddot(p, p)));
    if (s.type == 0) s.boundingRadius = std::sqrt(ddot(s.center, s.center)) + s.size.x;
    if (s.type == 2) s.boundingRadius = std::sqrt(ddot(s.center, s.center)) + s.size.x + s.size.y;
  }
  if (version == 2) {
    int count = -1;
    in >> count;
    if (count < 0 || count > maxPairs) throw std::runtime_error("Invalid body collision pair count");
    for (int k = 0; k < count; ++k) {
      ParsedModel::Pair p;
      in >> p.a >> p.b >> p.friction;
      if (p.a < 0 || p.a >= ns || p.b <= p.a || p.b >= ns ||
          m.shapes[p.a].body == m.shapes[p.b].body || p.friction < 0 || !std::isfinite(p.friction))
        throw std::runtime_error("Invalid body collision pair");
      for (auto old : m.pairs)
        if (old.a == p.a && old.b == p.b) throw std::runtime_error("Duplicate body collision pair");
      m.pairs.push_back(p);
    }
  }
  if (!in) throw std::runtime_error("Truncated model");
  std::string extra;
  if (in >> extra) throw std::runtime_error("Unexpected model data");
  return m;
}

template <class R> struct HostModel {
  DevModel<R> dev{};
  std::vector<R> points;   // [npoints][3]
  std::vector<std::string> jointNames;
};

template <class R>
HostModel<R> convertModel(const ParsedModel &o, double dt, int iterations, bool specialized,
                          int maxPairs = kReferencePairs) {
  auto require = [](bool c, const char *msg) { if (!c) throw std::invalid_argument(msg); };
  require(o.bodies.size() <= 32 && o.joints.size() <= 32 && o.shapes.size() <= 32 &&
              int(o.pairs.size()) <= std::min(maxPairs, kMaxPairs),
          "CUDA model capacity exceeded (32 bodies/joints/shapes)");
  require(o.bodies.size() > 1, "CUDA batch needs at least one body");
  const int contactCapacity = specialized ? 64 : 160;
  if (specialized)
    require(o.bodies.size() <= 16 && o.joints.size() <= 14, "Model exceeds selected state body/joint capacity");
  int bound = int(o.pairs.size()), groundCap = 0;
  if (o.ground)
    for (const auto &s : o.shapes)
      if (s.ground && o.bodies[s.body].mass > 0) {
        bound += 4;
        int points = s.type == 0 ? 1 : (s.type == 2 ? 2 : int(s.localPoints.size()));
        groundCap += std::min(4, points);
      }
  require(bound <= contactCapacity, "Model exceeds selected state contact capacity");

  HostModel<R> h;
  DevModel<R> &d = h.dev;
  d.nb = int(o.bodies.size());
  d.nj = int(o.joints.size());
  d.ns = int(o.shapes.size());
  d.np = int(o.pairs.size());
  d.bound = bound;
  d.groundCap = groundCap;
  d.ground = o.ground;
  d.iterations = iterations;
  d.dt = R(dt);
  d.alpha = R(0.9);
  d.gamma = R(0.99);
  d.betaLinear = R(1e7);
  d.betaAngular = R(1e5);
  // FP32 has an attainable stopping tolerance (model.hpp:358-359).
  d.tolerance = std::is_same_v<R, float> ? R(1e-6) : R(1e-7);
  d.gravity[0] = R(o.gravity.x); d.gravity[1] = R(o.gravity.y); d.gravity[2] = R(o.gravity.z);
  auto set3 = [](R *dst, DVec v) { dst[0] = R(v.x); dst[1] = R(v.y); dst[2] = R(v.z); };
  auto set4 = [](R *dst, DQuat q) { dst[0] = R(q.w); dst[1] = R(q.x); dst[2] = R(q.y); dst[3] = R(q.z); };
  for (int i = 0; i < d.nb; ++i) {
    const auto &b = o.bodies[i];
    d.mass[i] = R(b.mass);
    set3(d.inertia[i], b.inertia); set3(d.x[i], b.x); set4(d.q[i], b.q); set3(d.v[i], b.v); set3(d.w[i], b.w);
    d.color[i] = 0;
  }
  std::vector<int> incoming(d.nb, 0);
  for (auto &j : o.joints) require(++incoming[j.b] == 1, "A body must have at most one parent hinge");
  std::vector<bool> seen(d.nb);
  for (int i = 0; i < d.nb; ++i) seen[i] = incoming[i] == 0;
  for (int i = 0; i < d.nj; ++i) {
    const auto &j = o.joints[i];
    require(j.a < j.b, "CUDA reset requires topological body ordering");
    require(seen[j.a], "Joint list must follow parent-before-child ordering");
    seen[j.b] = true;
    d.ja[i] = j.a; d.jb[i] = j.b;
    d.color[j.b] = 1 - d.color[j.a];
    set3(d.ra[i], j.ra); set3(d.rb[i], j.rb); set3(d.axisA[i], j.axisA); set3(d.axisB[i], j.axisB);
    set3(d.tangentA[i], j.tangentA); set3(d.tangentB[i], j.tangentB);
    d.lo[i] = R(j.lo); d.hi[i] = R(j.hi); d.limited[i] = j.limited; d.damping[i] = R(j.damping);
    d.armature[i] = R(j.armature); d.frictionloss[i] = R(j.frictionloss); d.torque[i] = R(j.torque);
    d.kp[i] = R(j.kp); d.target[i] = R(j.target); d.maxTorque[i] = R(j.maxTorque);
    d.jInfo[i][0] = j.a; d.jInfo[i][1] = j.b; d.jInfo[i][2] = j.limited; d.jInfo[i][3] = 0;
    for (int k = 0; k < 3; ++k) {
      d.jFrame[i][k] = d.ra[i][k]; d.jFrame[i][3 + k] = d.rb[i][k]; d.jFrame[i][6 + k] = d.axisA[i][k];
      d.jFrame[i][9 + k] = d.axisB[i][k]; d.jFrame[i][12 + k] = d.tangentA[i][k]; d.jFrame[i][15 + k] = d.tangentB[i][k];
    }
    d.jFrame[i][18] = d.lo[i]; d.jFrame[i][19] = d.hi[i];
    h.jointNames.push_back(j.name);
  }
  for (auto &j : o.joints)
    require(o.bodies[j.a].mass == 0 || o.bodies[j.b].mass == 0 || d.color[j.a] != d.color[j.b],
            "Joint graph must be bipartite");
  if (specialized) {
    require(d.nb == 16 && d.nj == 14, "MicroDuck specialized backend requires 16 bodies and 14 hinges");
    const char *expected[] = {"left_hip_yaw", "left_hip_roll", "left_hip_pitch", "left_knee",
                              "left_ankle", "neck_pitch", "head_pitch", "head_yaw", "head_roll",
                              "right_hip_yaw", "right_hip_roll", "right_hip_pitch", "right_knee",
                              "right_ankle"};
    for (int i = 0; i < 14; ++i) {
      std::string name = h.jointNames[i];
      if (name.rfind("robot/", 0) == 0) name = name.substr(6);
      require(name == expected[i], "Unsupported MicroDuck joint layout");
    }
  }
  int adjacency = 0;
  for (int bi = 0; bi < d.nb; ++bi) {
    d.csrOffset[bi] = adjacency;
    for (int ji = 0; ji < d.nj; ++ji)
      if (d.ja[ji] == bi || d.jb[ji] == bi) d.csrJoint[adjacency++] = ji;
  }
  d.csrOffset[d.nb] = adjacency;
  int fill = 0;
  d.colorMax = 1;
  for (int c = 0; c < 2; ++c) {
    d.colorStart[c] = fill;
    for (int bi = 0; bi < d.nb; ++bi)
      if (d.color[bi] == c && d.mass[bi] > R(0)) d.colorBody[fill++] = bi;
    d.colorMax = std::max(d.colorMax, fill - d.colorStart[c]);
  }
  d.colorStart[2] = fill;
  for (int i = 0; i < d.ns; ++i) {
    const auto &s = o.shapes[i];
    d.sBody[i] = s.body; d.sType[i] = s.type; d.sGround[i] = s.ground;
    set3(d.sCenter[i], s.center); set3(d.sSize[i], s.size); set4(d.sQ[i], s.q);
    d.sFriction[i] = R(s.friction); d.sRadius[i] = R(s.boundingRadius);
    d.sOffset[i] = int(h.points.size() / 3);
    d.sCount[i] = s.type == 0 ? 1 : (s.type == 2 ? 2 : int(s.localPoints.size()));
    // Warm-start keys pack (shape, point) into 10 + 20 bits.
    if (d.sCount[i] >= (1 << 20)) throw std::invalid_argument("Collision shape has too many points");
    DVec interior = s.center;
    if (!s.localPoints.empty()) {
      interior = {};
      for (auto p : s.localPoints) interior = dadd(interior, p);
      interior = dscale(interior, 1 / double(s.localPoints.size()));
    }
    set3(d.sInterior[i], interior);
    for (auto p : s.localPoints) {
      h.points.push_back(R(p.x)); h.points.push_back(R(p.y)); h.points.push_back(R(p.z));
    }
  }
  for (int i = 0; i < d.np; ++i) {
    d.pA[i] = o.pairs[i].a; d.pB[i] = o.pairs[i].b; d.pFriction[i] = R(o.pairs[i].friction);
  }
  return h;
}

}  // namespace duckb200
