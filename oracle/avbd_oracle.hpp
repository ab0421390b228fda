// CPU restatement of the duck_gym AVBD environment step -- TEST
// INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and bench.py's
// cpu_baseline leg may load this code, and only as the checker.  The product
// (duck_gym_b200/csrc) never links it.
//
// This file restates, in scalar C++, the algorithm of the reference's shared
// solver core (src/cuda/kernel.cuh, src/cuda/convex.cuh, src/cuda/model.hpp
// and the .duck loader of src/solver.cpp).  Each function cites the lines it
// follows.  The floating-point operations are kept in the reference's order,
// including the places where the reference's float build silently promotes to
// double, so that a build with -ffp-contract=off reproduces the reference CPU
// twin (_duck_reference.CpuBatch32/64) bit for bit; tests check exactly that.
//
// Template parameters: R is the solver scalar (float or double); W is the
// wide type used where the reference promotes (double).  A counting scalar
// (Tally, below) can be substituted for both to count the algorithmic
// floating-point operations of a run.
#pragma once
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <fstream>
#include <limits>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

namespace avbd_oracle {

// ---------------------------------------------------------------------------
// Operation counting scalar.
struct OpCounts {
  uint64_t add = 0, mul = 0, div = 0, sqrt = 0, sin = 0, cos = 0, tan = 0,
           atan2 = 0, hypot = 0, rem = 0;
};
inline OpCounts &counts() {
  static thread_local OpCounts c;
  return c;
}
template <class T> struct Tally {
  T v{};
  Tally() = default;
  Tally(T x) : v(x) {}
  template <class U, class = std::enable_if_t<std::is_arithmetic_v<U>>>
  Tally(U x) : v(T(x)) {}
  template <class U> explicit Tally(Tally<U> o) : v(T(o.v)) {}
  explicit operator T() const { return v; }
};
template <class T> Tally<T> operator+(Tally<T> a, Tally<T> b) { ++counts().add; return a.v + b.v; }
template <class T> Tally<T> operator-(Tally<T> a, Tally<T> b) { ++counts().add; return a.v - b.v; }
template <class T> Tally<T> operator*(Tally<T> a, Tally<T> b) { ++counts().mul; return a.v * b.v; }
template <class T> Tally<T> operator/(Tally<T> a, Tally<T> b) { ++counts().div; return a.v / b.v; }
template <class T> Tally<T> operator-(Tally<T> a) { return -a.v; }
template <class T> Tally<T> &operator+=(Tally<T> &a, Tally<T> b) { return a = a + b; }
template <class T> Tally<T> &operator-=(Tally<T> &a, Tally<T> b) { return a = a - b; }
template <class T> Tally<T> &operator*=(Tally<T> &a, Tally<T> b) { return a = a * b; }
template <class T> Tally<T> &operator/=(Tally<T> &a, Tally<T> b) { return a = a / b; }
template <class T> bool operator<(Tally<T> a, Tally<T> b) { return a.v < b.v; }
template <class T> bool operator>(Tally<T> a, Tally<T> b) { return a.v > b.v; }
template <class T> bool operator<=(Tally<T> a, Tally<T> b) { return a.v <= b.v; }
template <class T> bool operator>=(Tally<T> a, Tally<T> b) { return a.v >= b.v; }
template <class T> bool operator==(Tally<T> a, Tally<T> b) { return a.v == b.v; }
template <class T> bool operator!=(Tally<T> a, Tally<T> b) { return a.v != b.v; }

template <class T> struct Raw { using type = T; };
template <class T> struct Raw<Tally<T>> { using type = T; };
template <class T> typename Raw<T>::type raw(T x) {
  if constexpr (std::is_arithmetic_v<T>) return x; else return x.v;
}
// Math entry points; each is one counted operation for a Tally argument.
template <class T> T m_sqrt(T x) {
  if constexpr (std::is_arithmetic_v<T>) return std::sqrt(x);
  else { ++counts().sqrt; return std::sqrt(x.v); }
}
template <class T> T m_sin(T x) {
  if constexpr (std::is_arithmetic_v<T>) return std::sin(x);
  else { ++counts().sin; return std::sin(x.v); }
}
template <class T> T m_cos(T x) {
  if constexpr (std::is_arithmetic_v<T>) return std::cos(x);
  else { ++counts().cos; return std::cos(x.v); }
}
template <class T> T m_tan(T x) {
  if constexpr (std::is_arithmetic_v<T>) return std::tan(x);
  else { ++counts().tan; return std::tan(x.v); }
}
template <class T> T m_atan2(T y, T x) {
  if constexpr (std::is_arithmetic_v<T>) return std::atan2(y, x);
  else { ++counts().atan2; return std::atan2(y.v, x.v); }
}
template <class T> T m_hypot(T x, T y) {
  if constexpr (std::is_arithmetic_v<T>) return std::hypot(x, y);
  else { ++counts().hypot; return std::hypot(x.v, y.v); }
}
template <class T> T m_remainder(T x, T y) {
  if constexpr (std::is_arithmetic_v<T>) return std::remainder(x, y);
  else { ++counts().rem; return std::remainder(x.v, y.v); }
}
template <class T> T m_abs(T x) {
  if constexpr (std::is_arithmetic_v<T>) return std::abs(x); else return std::abs(x.v);
}
template <class T> bool m_finite(T x) { return std::isfinite(raw(x)); }
template <class T> T m_nan() { return T(std::numeric_limits<typename Raw<T>::type>::quiet_NaN()); }

// ---------------------------------------------------------------------------
// Small vector algebra (kernel.cuh:37-60, 86-163).
template <class R> struct V3 {
  R x{}, y{}, z{};
  R &operator[](int i) { return i == 0 ? x : (i == 1 ? y : z); }
  R operator[](int i) const { return i == 0 ? x : (i == 1 ? y : z); }
};
template <class R> struct Q4 { R w = R(1), x{}, y{}, z{}; };

template <class R> R rmin(R a, R b) { return a < b ? a : b; }         // kernel.cuh:37
template <class R> R rmax(R a, R b) { return a > b ? a : b; }         // kernel.cuh:38
template <class R> R rclamp(R v, R a, R b) { return rmin(rmax(v, a), b); }

template <class R> V3<R> operator+(V3<R> a, V3<R> b) { return {a.x + b.x, a.y + b.y, a.z + b.z}; }
template <class R> V3<R> operator-(V3<R> a, V3<R> b) { return {a.x - b.x, a.y - b.y, a.z - b.z}; }
template <class R> V3<R> operator-(V3<R> a) { return {-a.x, -a.y, -a.z}; }
template <class R> V3<R> scaled(V3<R> a, R s) { return {a.x * s, a.y * s, a.z * s}; }
// Vec3 / s multiplies by the reciprocal (kernel.cuh:100).
template <class R> V3<R> divided(V3<R> a, R s) { return scaled(a, R(1) / s); }
template <class R> R dot(V3<R> a, V3<R> b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
template <class R> V3<R> cross(V3<R> a, V3<R> b) {
  return {a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x};
}
template <class R, class W> R norm(V3<R> a) { return m_sqrt(dot(a, a)); }
template <class R, class W> V3<R> unit(V3<R> a) {   // kernel.cuh:110-115
  R n = norm<R, W>(a);
  if (W(n) < W(1e-15)) return {m_nan<R>(), m_nan<R>(), m_nan<R>()};
  return divided(a, n);
}
template <class R> Q4<R> conj(Q4<R> q) { return {q.w, -q.x, -q.y, -q.z}; }
template <class R> Q4<R> qmul(Q4<R> a, Q4<R> b) {   // kernel.cuh:120-125
  return {a.w * b.w - a.x * b.x - a.y * b.y - a.z * b.z,
          a.w * b.x + a.x * b.w + a.y * b.z - a.z * b.y,
          a.w * b.y - a.x * b.z + a.y * b.w + a.z * b.x,
          a.w * b.z + a.x * b.y - a.y * b.x + a.z * b.w};
}
template <class R, class W> Q4<R> qnormalized(Q4<R> q) {   // kernel.cuh:126-131
  R n = m_sqrt(q.w * q.w + q.x * q.x + q.y * q.y + q.z * q.z);
  if (W(n) < W(1e-15)) return {m_nan<R>(), m_nan<R>(), m_nan<R>(), m_nan<R>()};
  return {q.w / n, q.x / n, q.y / n, q.z / n};
}
template <class R> V3<R> rotate(Q4<R> q, V3<R> v) {   // kernel.cuh:132-135
  V3<R> u{q.x, q.y, q.z};
  return v + scaled(cross(u, cross(u, v) + scaled(v, q.w)), R(2));
}
// Exponential map; the small-angle branch is evaluated in double by the
// reference (kernel.cuh:136-145).
template <class R, class W> Q4<R> qexp(V3<R> v) {
  R a = norm<R, W>(v);
  R s = W(a) < W(1e-8) ? R(W(0.5) - W(a * a / R(48))) : m_sin(a / R(2)) / a;
  return qnormalized<R, W>({m_cos(a / R(2)), s * v.x, s * v.y, s * v.z});
}
template <class R, class W> V3<R> qlog(Q4<R> q) {   // kernel.cuh:146-153
  q = qnormalized<R, W>(q);
  if (q.w < R(0)) q = {-q.w, -q.x, -q.y, -q.z};
  V3<R> v{q.x, q.y, q.z};
  R s = norm<R, W>(v);
  return scaled(v, W(s) < W(1e-10) ? R(2) : R(2) * m_atan2(s, q.w) / s);
}
// remainder(a, 2 pi) in double (kernel.cuh:154-160).
template <class R, class W> R wrap(R a) {
  return R(m_remainder(W(a), W(2) * W(std::acos(-1.0))));
}

template <class R> struct V6 { R v[6]{}; R &operator[](int i) { return v[i]; } R operator[](int i) const { return v[i]; } };
template <class R> struct M6 { V6<R> r[6]{}; V6<R> &operator[](int i) { return r[i]; } const V6<R> &operator[](int i) const { return r[i]; } };
template <class R> V6<R> row6(V3<R> t, V3<R> r) { return {{t.x, t.y, t.z, r.x, r.y, r.z}}; }
// Rank-one Gauss-Newton stamp (kernel.cuh:164-176).
template <class R> void stamp(M6<R> &H, V6<R> &g, const V6<R> &J, R force, R stiffness) {
  for (int i = 0; i < 6; ++i) {
    g[i] += J[i] * force;
    for (int j = 0; j < 6; ++j) H[i][j] += stiffness * J[i] * J[j];
  }
}
// 6x6 Cholesky solve of H x = -g; NaN on a non-positive pivot (kernel.cuh:177-228).
template <class R> V6<R> solve6(const M6<R> &H, const V6<R> &g) {
  M6<R> L{};
  for (int i = 0; i < 6; ++i)
    for (int j = 0; j <= i; ++j) {
      R v = H[i][j];
      for (int k = 0; k < j; ++k) v -= L[i][k] * L[j][k];
      if (i == j) {
        if (!(v > R(0)) || !m_finite(v)) {
          V6<R> bad;
          for (int k = 0; k < 6; ++k) bad[k] = m_nan<R>();
          return bad;
        }
        L[i][j] = m_sqrt(v);
      } else
        L[i][j] = v / L[j][j];
    }
  V6<R> y{}, x{};
  for (int i = 0; i < 6; ++i) {
    y[i] = -g[i];
    for (int k = 0; k < i; ++k) y[i] -= L[i][k] * y[k];
    y[i] /= L[i][i];
  }
  for (int i = 5; i >= 0; --i) {
    x[i] = y[i];
    for (int k = i + 1; k < 6; ++k) x[i] -= L[k][i] * x[k];
    x[i] /= L[i][i];
  }
  return x;
}

// ---------------------------------------------------------------------------
// Model and per-environment state (kernel.cuh:229-334, 365-382).
template <class R> struct Body {
  R mass{};
  V3<R> inertia{}, x{}, v{}, w{}, x0{}, xp{}, force{};
  Q4<R> q{}, q0{}, qp{};
};
template <class R> struct Joint {
  int a = 0, b = 0;
  V3<R> ra{}, rb{}, axisA{}, axisB{}, tangentA{}, tangentB{};
  R lo{}, hi{}, damping{}, armature{}, frictionloss{}, lambdaF{}, penaltyF = R(1),
      torque{}, kp{}, target{}, maxTorque{};
  bool limited = false;
  R angle0{}, velocity0{};
  R lambda[7]{}, penalty[7]{}, c0[7]{};
};
template <class R> struct Shape {
  int body = 0, type = 0, offset = 0, count = 0;
  bool ground = true;
  V3<R> center{}, size{}, interior{};
  Q4<R> q{};
  R friction = R(.8), boundingRadius{};
};
template <class R> struct Pair { int a = 0, b = 0; R friction{}; };
template <class R> struct Contact {
  int body = 0, shape = 0, feature = 0, other = -1, otherShape = -1;
  V3<R> local{}, anchor{}, localB{};
  V3<R> tangent1{R(1), R(0), R(0)}, tangent2{R(0), R(1), R(0)}, normal{R(0), R(0), R(1)};
  R friction{}, c0{};
  R lambda[3]{}, penalty[3]{};
  bool stick = false;
};
template <class R> struct Options {
  R dt = R(0.001), alpha = R(0.9), gamma = R(0.99), betaLinear = R(1e7),
    betaAngular = R(1e5), tolerance = R(1e-7);
  int iterations = 100;
  V3<R> gravity{R(0), R(0), R(-9.81)};
  bool ground = false;
};
template <class R> struct Diagnostics {
  R jointError{}, axisError{}, penetration{}, update{};
  int contacts = 0, iterations = 0;
  bool converged = false;
};
template <class R> struct Model {
  std::vector<Body<R>> bodies;
  std::vector<Joint<R>> joints;
  std::vector<Shape<R>> shapes;
  std::vector<Pair<R>> pairs;
  std::vector<V3<R>> points;
  Options<R> options;
  std::vector<int> colors, csrOffsets, csrJoints;
  std::vector<std::string> jointNames;
  int contactCapacity = 160;
};

template <class R> R minimumPenalty(int k) { return k < 3 ? R(1000) : R(1); }   // kernel.cuh:302
template <class R> R maximumPenalty(int k) { return k < 3 ? R(1e9) : R(1e7); }  // kernel.cuh:303

// ---------------------------------------------------------------------------
// .duck text loader (src/solver.cpp:67-174) and conversion to the solver
// model (src/cuda/model.hpp:237-360).  Loading runs in double like the
// reference; conversion rounds to R.
struct DModel {
  struct B { std::string name; double mass = 0; V3<double> inertia, x, v, w; Q4<double> q; };
  struct J {
    std::string name; int a = 0, b = 0;
    V3<double> ra, rb, axisA, axisB, tangentA, tangentB;
    bool limited = false;
    double lo = 0, hi = 0, damping = 0, armature = 0, frictionloss = 0, torque = 0,
           kp = 0, target = 0, maxTorque = 0;
  };
  struct S {
    int body = 0, type = 0; V3<double> center, size; Q4<double> q;
    double friction = 0.8; std::vector<V3<double>> vertices, localPoints;
    double boundingRadius = 0; bool ground = true;
  };
  struct P { int a = 0, b = 0; double friction = 0; };
  V3<double> gravity{0, 0, -9.81};
  bool ground = false;
  std::vector<B> bodies;
  std::vector<J> joints;
  std::vector<S> shapes;
  std::vector<P> pairs;
};

inline V3<double> dunit(V3<double> a) {
  double n = std::sqrt(dot(a, a));
  if (n < 1e-15) throw std::runtime_error("Zero direction");
  return divided(a, n);
}
inline Q4<double> dnormalized(Q4<double> q) {
  double n = std::sqrt(q.w * q.w + q.x * q.x + q.y * q.y + q.z * q.z);
  if (n < 1e-15) throw std::runtime_error("Zero quaternion");
  return {q.w / n, q.x / n, q.y / n, q.z / n};
}

// maxPairs: the reference rejects more than 32 body-collision pairs
// (solver.cpp:151-152); larger limits restate the same algorithm with a raised
// capacity, the checker of the library's pair-limit extension.
inline DModel loadDuck(const std::string &path, int maxPairs = 32) {
  std::ifstream in(path);
  if (!in) throw std::runtime_error("Cannot read model: " + path);
  DModel m;
  auto readV = [&] { V3<double> v; in >> v.x >> v.y >> v.z; return v; };
  auto readQ = [&] { Q4<double> q; in >> q.w >> q.x >> q.y >> q.z; return dnormalized(q); };
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
    j.axisA = dunit(readV()); j.axisB = dunit(readV());
    j.tangentA = dunit(readV()); j.tangentB = dunit(readV());
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
    for (int k = 0; k < n; ++k) s.vertices.push_back(readV());
    if (version == 2) in >> s.ground;
    if (s.type == 3 && n < 4) throw std::runtime_error("Convex mesh needs at least four vertices");
    if (s.type == 1) {
      for (int i = 0; i < 8; ++i)
        s.localPoints.push_back(s.center + rotate(s.q, V3<double>{(i & 1 ? 1 : -1) * s.size.x,
                                                                  (i & 2 ? 1 : -1) * s.size.y,
                                                                  (i & 4 ? 1 : -1) * s.size.z}));
    } else if (s.type == 3) {
      for (auto v : s.vertices) s.localPoints.push_back(s.center + rotate(s.q, v));
    }
    for (auto p : s.localPoints) s.boundingRadius = std::max(s.boundingRadius, std::sqrt(dot(p, p)));
    if (s.type == 0) s.boundingRadius = std::sqrt(dot(s.center, s.center)) + s.size.x;
    if (s.type == 2) s.boundingRadius = std::sqrt(dot(s.center, s.center)) + s.size.x + s.size.y;
  }
  if (version == 2) {
    int count = -1;
    in >> count;
    if (count < 0 || count > maxPairs) throw std::runtime_error("Invalid body collision pair count");
    for (int k = 0; k < count; ++k) {
      DModel::P p;
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

template <class R> V3<R> toR(V3<double> v) { return {R(v.x), R(v.y), R(v.z)}; }
template <class R> Q4<R> toR(Q4<double> q) { return {R(q.w), R(q.x), R(q.y), R(q.z)}; }

// model.hpp:237-360.  contactCapacity is 160 for the generic state and 64 for
// the compact MicroDuck state (kernel.cuh:1097-1098).
template <class R>
Model<R> convertModel(const DModel &o, double dt, int iterations, int contactCapacity,
                      int bodyCapacity = 32, int jointCapacity = 32, int maxPairs = 32) {
  auto require = [](bool c, const char *m) { if (!c) throw std::invalid_argument(m); };
  require(o.bodies.size() <= 32 && o.joints.size() <= 32 && o.shapes.size() <= 32 &&
              int(o.pairs.size()) <= maxPairs,
          "CUDA model capacity exceeded (32 bodies/joints/shapes)");
  require(o.bodies.size() > 1, "CUDA batch needs at least one body");
  require(int(o.bodies.size()) <= bodyCapacity && int(o.joints.size()) <= jointCapacity,
          "Model exceeds selected state body/joint capacity");
  size_t maximumContacts = o.pairs.size();
  if (o.ground)
    for (const auto &s : o.shapes)
      if (s.ground && o.bodies[s.body].mass > 0) maximumContacts += 4;
  require(int(maximumContacts) <= contactCapacity, "Model exceeds selected state contact capacity");
  Model<R> m;
  m.contactCapacity = contactCapacity;
  m.bodies.resize(o.bodies.size());
  for (size_t i = 0; i < o.bodies.size(); ++i) {
    auto &d = m.bodies[i];
    auto &b = o.bodies[i];
    d.mass = R(b.mass); d.inertia = toR<R>(b.inertia); d.x = toR<R>(b.x);
    d.v = toR<R>(b.v); d.w = toR<R>(b.w); d.q = toR<R>(b.q);
  }
  m.colors.assign(o.bodies.size(), 0);
  std::vector<int> incoming(o.bodies.size(), 0);
  for (auto &j : o.joints) require(++incoming[j.b] == 1, "A body must have at most one parent hinge");
  std::vector<bool> seen(o.bodies.size());
  for (size_t i = 0; i < seen.size(); ++i) seen[i] = incoming[i] == 0;
  m.joints.resize(o.joints.size());
  for (size_t i = 0; i < o.joints.size(); ++i) {
    auto &d = m.joints[i];
    auto &j = o.joints[i];
    require(j.a < j.b, "CUDA reset requires topological body ordering");
    require(seen[j.a], "Joint list must follow parent-before-child ordering");
    seen[j.b] = true;
    d.a = j.a; d.b = j.b;
    m.colors[j.b] = 1 - m.colors[j.a];
    d.ra = toR<R>(j.ra); d.rb = toR<R>(j.rb); d.axisA = toR<R>(j.axisA); d.axisB = toR<R>(j.axisB);
    d.tangentA = toR<R>(j.tangentA); d.tangentB = toR<R>(j.tangentB);
    d.lo = R(j.lo); d.hi = R(j.hi); d.limited = j.limited; d.damping = R(j.damping);
    d.armature = R(j.armature); d.frictionloss = R(j.frictionloss); d.torque = R(j.torque);
    d.kp = R(j.kp); d.target = R(j.target); d.maxTorque = R(j.maxTorque);
    for (int k = 0; k < 7; ++k) d.penalty[k] = R(k < 3 ? 1000.0 : 1.0);
    m.jointNames.push_back(j.name);
  }
  for (auto &j : o.joints)
    require(o.bodies[j.a].mass == 0 || o.bodies[j.b].mass == 0 || m.colors[j.a] != m.colors[j.b],
            "Joint graph must be bipartite");
  m.csrOffsets.assign(o.bodies.size() + 1, 0);
  for (size_t bi = 0; bi < o.bodies.size(); ++bi) {
    m.csrOffsets[bi] = int(m.csrJoints.size());
    for (size_t ji = 0; ji < o.joints.size(); ++ji)
      if (o.joints[ji].a == int(bi) || o.joints[ji].b == int(bi)) m.csrJoints.push_back(int(ji));
  }
  m.csrOffsets[o.bodies.size()] = int(m.csrJoints.size());
  m.shapes.resize(o.shapes.size());
  for (size_t i = 0; i < o.shapes.size(); ++i) {
    auto &d = m.shapes[i];
    auto &s = o.shapes[i];
    d.body = s.body; d.ground = s.ground; d.type = s.type;
    d.center = toR<R>(s.center); d.size = toR<R>(s.size); d.q = toR<R>(s.q);
    d.friction = R(s.friction); d.boundingRadius = R(s.boundingRadius);
    d.offset = int(m.points.size());
    d.count = s.type == 0 ? 1 : (s.type == 2 ? 2 : int(s.localPoints.size()));
    V3<double> interior = s.center;
    if (!s.localPoints.empty()) {
      interior = {};
      for (auto p : s.localPoints) interior = interior + p;
      interior = divided(interior, double(s.localPoints.size()));
    }
    d.interior = toR<R>(interior);
    for (auto p : s.localPoints) m.points.push_back(toR<R>(p));
  }
  for (auto &p : o.pairs) m.pairs.push_back({p.a, p.b, R(p.friction)});
  m.options.dt = R(dt);
  m.options.iterations = iterations;
  m.options.gravity = toR<R>(o.gravity);
  m.options.ground = o.ground;
  // FP32 has an attainable stopping tolerance (model.hpp:358-359).
  m.options.tolerance = std::is_same_v<typename Raw<R>::type, float> ? R(1e-6) : R(1e-7);
  return m;
}

// ---------------------------------------------------------------------------
// Convex narrow phase: minimum portal refinement (convex.cuh:9-217).
template <class R> struct Support { V3<R> v{}, a{}, b{}; };
template <class R> struct ConvexHit { int status = 0; V3<R> normal{}, position{}; R depth{}; };

template <class R, class W>
V3<R> shapeSupport(const Shape<R> &s, const Body<R> &b, const V3<R> *points, V3<R> d, R inflation) {
  V3<R> ld = rotate(conj(b.q), d), local{};
  if (s.type == 0 || s.type == 2) {
    local = s.center + scaled(unit<R, W>(ld), s.size.x);
    if (s.type == 2) {
      V3<R> axis = rotate(s.q, V3<R>{R(0), R(0), R(1)});
      local = local + scaled(axis, dot(axis, ld) >= R(0) ? s.size.y : -s.size.y);
    }
  } else {
    int best = -1;
    R value = R(-INFINITY);
    for (int i = 0; i < s.count; ++i) {
      R c = dot(points[s.offset + i], ld);
      if (c > value) { best = i; value = c; }
    }
    local = points[s.offset + best];
  }
  return b.x + rotate(b.q, local) + scaled(d, inflation);
}
template <class R, class W> struct Minkowski {
  const Shape<R> &sa, &sb;
  const Body<R> &a, &b;
  const V3<R> *points;
  R inflation;
  Support<R> support(V3<R> d) const {
    Support<R> p;
    p.a = shapeSupport<R, W>(sa, a, points, d, inflation / R(2));
    p.b = shapeSupport<R, W>(sb, b, points, -d, inflation / R(2));
    p.v = p.a - p.b;
    return p;
  }
};
template <class R, class W> V3<R> portalDirection(const Support<R> *p) {
  return unit<R, W>(cross(p[2].v - p[1].v, p[3].v - p[1].v));
}
template <class R> void expandPortal(Support<R> *p, const Support<R> &v) {
  V3<R> c = cross(v.v, p[0].v);
  if (dot(p[1].v, c) > R(0)) {
    if (dot(p[2].v, c) > R(0)) p[1] = v; else p[3] = v;
  } else if (dot(p[3].v, c) > R(0)) {
    p[2] = v;
  } else {
    p[1] = v;
  }
}
template <class R> R portalAdvance(const Support<R> *p, const Support<R> &v, V3<R> d) {
  return dot(v.v, d) - rmax(dot(p[1].v, d), rmax(dot(p[2].v, d), dot(p[3].v, d)));
}
template <class R> V3<R> closestTriangleOrigin(V3<R> a, V3<R> b, V3<R> c) {
  V3<R> best = a;
  R distance = dot(a, a);
  V3<R> v[3] = {a, b, c};
  for (int i = 0; i < 3; ++i) {
    V3<R> start = v[i], edge = v[(i + 1) % 3] - start;
    R square = dot(edge, edge);
    V3<R> point = start + scaled(edge, square > R(0) ? rclamp(-dot(start, edge) / square, R(0), R(1)) : R(0));
    if (dot(point, point) < distance) { distance = dot(point, point); best = point; }
  }
  V3<R> ab = b - a, ac = c - a, n = cross(ab, ac);
  R nn = dot(n, n);
  if (nn > R(0)) {
    V3<R> point = scaled(n, dot(n, a) / nn);
    R u = dot(cross(b - point, c - point), n) / nn;
    R w = dot(cross(c - point, a - point), n) / nn;
    if (u >= R(0) && w >= R(0) && u + w <= R(1) && dot(point, point) < distance) best = point;
  }
  return best;
}
template <class R> V3<R> portalPosition(const Support<R> *p, V3<R> d) {
  R w[4] = {dot(cross(p[1].v, p[2].v), p[3].v), dot(cross(p[3].v, p[2].v), p[0].v),
            dot(cross(p[0].v, p[1].v), p[3].v), dot(cross(p[2].v, p[1].v), p[0].v)};
  R sum = w[0] + w[1] + w[2] + w[3];
  if (!(sum > R(0))) {
    w[0] = R(0);
    w[1] = dot(cross(p[2].v, p[3].v), d);
    w[2] = dot(cross(p[3].v, p[1].v), d);
    w[3] = dot(cross(p[1].v, p[2].v), d);
    sum = w[1] + w[2] + w[3];
  }
  if (!(sum > R(0))) return {m_nan<R>(), m_nan<R>(), m_nan<R>()};
  V3<R> position{};
  for (int i = 0; i < 4; ++i) position = position + scaled(p[i].a + p[i].b, w[i] / (R(2) * sum));
  return position;
}
template <class R, class W> ConvexHit<R> convexContact(const Minkowski<R, W> &q, R tolerance) {
  ConvexHit<R> result;
  Support<R> p[4];
  p[0].a = q.a.x + rotate(q.a.q, q.sa.interior);
  p[0].b = q.b.x + rotate(q.b.q, q.sb.interior);
  p[0].v = p[0].a - p[0].b;
  R scale = rmax(R(.001), q.sa.boundingRadius + q.sb.boundingRadius);
  R epsilon = tolerance * R(.01);
  if (norm<R, W>(p[0].v) < epsilon) p[0].v.x += epsilon * R(10);
  V3<R> d = unit<R, W>(-p[0].v);
  p[1] = q.support(d);
  if (dot(p[1].v, d) <= R(0)) return result;
  d = cross(p[0].v, p[1].v);
  if (norm<R, W>(d) <= epsilon * scale) {
    result.status = 1;
    result.depth = norm<R, W>(p[1].v);
    result.normal = result.depth > epsilon ? -unit<R, W>(p[1].v) : unit<R, W>(p[0].v);
    result.position = divided(p[1].a + p[1].b, R(2));
    return result;
  }
  d = unit<R, W>(d);
  p[2] = q.support(d);
  if (dot(p[2].v, d) <= R(0)) return result;
  d = unit<R, W>(cross(p[1].v - p[0].v, p[2].v - p[0].v));
  if (dot(d, p[0].v) > R(0)) { std::swap(p[1], p[2]); d = -d; }
  bool discovered = false;
  for (int it = 0; it < 128; ++it) {
    if (!m_finite(d.x)) break;
    p[3] = q.support(d);
    if (dot(p[3].v, d) <= R(0)) return result;
    if (dot(cross(p[1].v, p[3].v), p[0].v) < -epsilon * scale * scale) p[2] = p[3];
    else if (dot(cross(p[3].v, p[2].v), p[0].v) < -epsilon * scale * scale) p[1] = p[3];
    else { discovered = true; break; }
    d = unit<R, W>(cross(p[1].v - p[0].v, p[2].v - p[0].v));
  }
  if (!discovered) { result.status = -1; return result; }
  bool intersecting = false;
  for (int it = 0; it < 128; ++it) {
    d = portalDirection<R, W>(p);
    if (!m_finite(d.x)) break;
    if (dot(d, p[1].v) >= -epsilon) { intersecting = true; break; }
    auto point = q.support(d);
    if (dot(point.v, d) < R(0) || portalAdvance(p, point, d) <= tolerance) return result;
    expandPortal(p, point);
  }
  if (!intersecting) { result.status = -1; return result; }
  for (int it = 0; it < 256; ++it) {
    d = portalDirection<R, W>(p);
    if (!m_finite(d.x)) break;
    auto point = q.support(d);
    if (portalAdvance(p, point, d) <= tolerance) {
      V3<R> closest = closestTriangleOrigin(p[1].v, p[2].v, p[3].v);
      result.depth = norm<R, W>(closest);
      result.normal = result.depth > epsilon ? divided(-closest, result.depth) : -d;
      result.position = portalPosition(p, d);
      result.status = m_finite(result.position.x) ? 1 : -1;
      return result;
    }
    expandPortal(p, point);
  }
  result.status = -1;
  return result;
}

// ---------------------------------------------------------------------------
// One environment (kernel.cuh:365-1096), executed serially.
template <class R, class W = double> struct Env {
  const Model<R> *model = nullptr;
  std::vector<Body<R>> bodies;
  std::vector<Joint<R>> joints;
  std::vector<Contact<R>> contacts, previous;
  std::vector<int> colors;
  int colorCount = 2;
  Options<R> options;
  Diagnostics<R> diagnostics;
  int failed = 0;

  void initialize(const Model<R> *m) {   // kernel.cuh:383-396
    model = m;
    options = m->options;
    bodies = m->bodies;
    joints = m->joints;
    contacts.clear();
    colors.assign(m->bodies.size(), 0);
    diagnostics = {};
    failed = 0;
  }
  // kernel.cuh:397-420
  template <class T> void resetPose(const T *q, const T *roots) {
    for (auto &b : bodies) { b.v = {}; b.w = {}; b.force = {}; }
    bodies[1].x = bodies[1].x + V3<R>{R(roots[0]), R(roots[1]), R(roots[2])};
    bodies[1].q = qmul(qexp<R, W>(V3<R>{R(roots[3]), R(roots[4]), R(roots[5])}), bodies[1].q);
    for (size_t i = 0; i < joints.size(); ++i) {
      auto &j = joints[i];
      const auto &oa = model->bodies[j.a];
      const auto &ob = model->bodies[j.b];
      V3<R> originalAxis = rotate(oa.q, j.axisA), t = rotate(oa.q, j.tangentA), u = rotate(ob.q, j.tangentB);
      R originalAngle = m_atan2(dot(originalAxis, cross(t, u)), dot(t, u));
      auto &a = bodies[j.a];
      auto &b = bodies[j.b];
      V3<R> axis = rotate(a.q, j.axisA);
      b.q = qnormalized<R, W>(qmul(qmul(qmul(qexp<R, W>(scaled(axis, R(q[i]) - originalAngle)), a.q), conj(oa.q)), ob.q));
      b.x = a.x + rotate(a.q, j.ra) - rotate(b.q, j.rb);
    }
  }
  // kernel.cuh:421-443
  void advance(int substeps) {
    Diagnostics<R> summary{};
    summary.converged = true;
    for (int k = 0; k < substeps; ++k) {
      step();
      if (failed) break;
      summary.jointError = rmax(summary.jointError, diagnostics.jointError);
      summary.axisError = rmax(summary.axisError, diagnostics.axisError);
      summary.penetration = rmax(summary.penetration, diagnostics.penetration);
      summary.contacts = int(raw(rmax(R(summary.contacts), R(diagnostics.contacts))));
      summary.converged = summary.converged && diagnostics.converged;
      summary.iterations += diagnostics.iterations;
    }
    diagnostics = summary;
  }
  // kernel.cuh:448-466
  template <class T> void setMotor(const T *motor, const T *force) {
    for (size_t i = 0; i < joints.size(); ++i) {
      auto &j = joints[i];
      for (int k = 0; k < 3; ++k)
        if (!std::isfinite(double(motor[3 * i + k]))) failed = 1;
      if (motor[3 * i + 1] < 0 || motor[3 * i + 2] < 0) failed = 1;
      j.kp = R(0);
      j.maxTorque = R(0);
      j.torque = R(motor[3 * i]);
      j.frictionloss = R(motor[3 * i + 1]);
      j.damping = R(motor[3 * i + 2]);
    }
    for (int k = 0; k < 3; ++k)
      if (!std::isfinite(double(force[k]))) failed = 1;
    bodies[1].force = {R(force[0]), R(force[1]), R(force[2])};
  }
  V3<R> contactWorld(const Contact<R> &c, V3<R> v) const {   // kernel.cuh:802-804
    return scaled(c.tangent1, v.x) + scaled(c.tangent2, v.y) + scaled(c.normal, v.z);
  }
  template <class T> void contactForces(T *out, bool groundOnly) const {   // kernel.cuh:467-480
    std::vector<R> acc(bodies.size() * 3, R(0));
    for (auto &c : contacts) {
      if (groundOnly && c.other >= 0) continue;
      V3<R> f = -contactWorld(c, {c.lambda[0], c.lambda[1], c.lambda[2]});
      for (int k = 0; k < 3; ++k) {
        acc[c.body * 3 + k] += f[k];
        if (c.other >= 0) acc[c.other * 3 + k] -= f[k];
      }
    }
    for (size_t i = 0; i < acc.size(); ++i) out[i] = T(raw(acc[i]));
  }
  // kernel.cuh:805-827
  void contactValues(const Contact<R> &c, V3<R> &C, V6<R> *J, int bi = -1) const {
    const auto &a = bodies[c.body];
    V3<R> ra = rotate(a.q, c.local), delta = a.x + ra - c.anchor;
    V3<R> r = ra;
    R sign = R(1);
    if (c.other >= 0) {
      const auto &b = bodies[c.other];
      V3<R> rb = rotate(b.q, c.localB);
      delta = a.x + ra - b.x - rb;
      if (bi == c.other) { r = rb; sign = R(-1); }
    }
    V3<R> basis[3] = {c.tangent1, c.tangent2, c.normal};
    for (int k = 0; k < 3; ++k) {
      C[k] = dot(delta, basis[k]);
      V3<R> e = scaled(basis[k], sign);
      J[k] = row6(e, cross(r, e));
    }
    C.z -= options.alpha * c.c0;
  }
  template <class T> void selfContactStats(T *out) const {   // kernel.cuh:481-493
    R o0 = R(0), o1 = R(0);
    for (const auto &c : contacts)
      if (c.other >= 0) {
        V3<R> C;
        V6<R> J[3];
        contactValues(c, C, J);
        R depth = rmax(R(0), -(C.z + options.alpha * c.c0));
        if (c.lambda[2] < R(-1e-5) || depth > R(1e-6)) o0 += R(1);
        o1 = rmax(o1, depth);
      }
    out[0] = T(raw(o0));
    out[1] = T(raw(o1));
  }
  template <class T> void contactCounts(T *out) const {   // kernel.cuh:494-498
    R o[2] = {R(0), R(0)};
    for (const auto &c : contacts) o[c.other < 0 ? 0 : 1] += R(1);
    out[0] = T(raw(o[0]));
    out[1] = T(raw(o[1]));
  }
  V3<R> inertiaMul(const Body<R> &b, V3<R> w, bool inverse = false) const {   // kernel.cuh:275-280
    V3<R> local = rotate(conj(b.q0), w);
    for (int k = 0; k < 3; ++k) local[k] *= inverse ? R(1) / b.inertia[k] : b.inertia[k];
    return rotate(b.q0, local);
  }
  // Diagonal majorizer of the rotational geometric stiffness; the entry is
  // formed in double (kernel.cuh:283-301).
  void geometric(M6<R> &H, V3<R> r, V3<R> f) const {
    R rf = dot(r, f);
    for (int col = 0; col < 3; ++col) {
      R sum = R(0);
      for (int row = 0; row < 3; ++row) {
        R a = R(W(0.5) * W(r[row] * f[col] + f[row] * r[col]) - W(row == col ? rf : R(0)));
        sum += a * a;
      }
      H[col + 3][col + 3] += m_sqrt(sum);
    }
  }
  // Friction-cone clamped contact force (kernel.cuh:304-315).
  V3<R> contactForce(V3<R> C, const Contact<R> &c) const {
    V3<R> f;
    for (int k = 0; k < 3; ++k) f[k] = c.lambda[k] + c.penalty[k] * C[k];
    f.z = rmin(f.z, R(0));
    R t = m_hypot(f.x, f.y), bound = -c.friction * f.z;
    if (t > bound && t > R(0)) {
      f.x *= bound / t;
      f.y *= bound / t;
    }
    return f;
  }
  // Hinge of joint j, all seven rows for both sides (kernel.cuh:725-761).
  R angle(const Joint<R> &j) const {
    const auto &a = bodies[j.a];
    const auto &b = bodies[j.b];
    V3<R> axis = rotate(a.q, j.axisA), t = rotate(a.q, j.tangentA), u = rotate(b.q, j.tangentB);
    return m_atan2(dot(axis, cross(t, u)), dot(t, u));
  }
  // side: 0 -> parent rows, 1 -> child rows, 2 -> values only.
  R evaluateJoint(const Joint<R> &j, R *C, V6<R> *J, int side) const {
    const auto &a = bodies[j.a];
    const auto &b = bodies[j.b];
    V3<R> ra = rotate(a.q, j.ra), rb = rotate(b.q, j.rb), d = a.x + ra - b.x - rb;
    for (int k = 0; k < 3; ++k) {
      V3<R> e{};
      e[k] = R(1);
      C[k] = d[k];
      if (side == 0) J[k] = row6(e, cross(ra, e));
      else if (side == 1) J[k] = row6(-e, -cross(rb, e));
    }
    V3<R> axis = rotate(a.q, j.axisA), axisB = rotate(b.q, j.axisB), t1 = rotate(a.q, j.tangentA),
          t2 = cross(axis, t1);
    for (int k = 3; k < 5; ++k) {
      V3<R> t = k == 3 ? t1 : t2;
      C[k] = dot(t, axisB);
      if (side == 0) J[k] = row6(V3<R>{}, cross(t, axisB));
      else if (side == 1) J[k] = row6(V3<R>{}, cross(axisB, t));
    }
    R q = angle(j);
    C[5] = q - j.lo;
    C[6] = j.hi - q;
    if (side == 0) { J[5] = row6(V3<R>{}, -axis); J[6] = row6(V3<R>{}, axis); }
    else if (side == 1) { J[5] = row6(V3<R>{}, axis); J[6] = row6(V3<R>{}, -axis); }
    return q;
  }
  V3<R> point(const Shape<R> &s, const Body<R> &b, int k) const {   // kernel.cuh:576-583
    if (s.type == 1 || s.type == 3) return model->points[s.offset + k];
    V3<R> down = rotate(conj(b.q), V3<R>{R(0), R(0), -s.size.x});
    if (s.type == 0) return s.center + down;
    return s.center + rotate(s.q, V3<R>{R(0), R(0), R(k ? 1 : -1) * s.size.y}) + down;
  }
  // Ground manifold picks and body-pair MPR contacts (kernel.cuh:338-364, 584-724).
  void detectContacts() {
    previous = contacts;
    contacts.clear();
    for (size_t bi = 0; bi < bodies.size(); ++bi) colors[bi] = model->colors[bi];
    colorCount = 2;
    const R dt = options.dt;
    for (size_t si = 0; si < model->shapes.size(); ++si) {
      const auto &s = model->shapes[si];
      const auto &b = bodies[s.body];
      if (!options.ground || !s.ground || b.mass == R(0)) continue;
      R low = rmin(b.x.z, b.x.z + dt * b.v.z + dt * dt * (options.gravity.z + b.force.z / b.mass));
      if (W(low - s.boundingRadius * (R(1) + dt * norm<R, W>(b.w))) >= W(.003)) continue;
      V3<R> chosen[4];
      int n = 0;
      for (int pick = 0; pick < 4; ++pick) {
        int best = -1;
        R lowest = R(INFINITY);
        for (int k = 0; k < s.count; ++k) {
          V3<R> local = point(s, b, k), world = b.x + rotate(b.q, local);
          V3<R> vel = b.v + cross(b.w, world - b.x);
          R z = rmin(world.z, world.z + dt * vel.z + dt * dt * (options.gravity.z + b.force.z / b.mass));
          if (W(z) >= W(.003) || z >= lowest) continue;
          bool duplicate = false;
          for (int c = 0; c < n; ++c)
            if (W(m_hypot(chosen[c].x - world.x, chosen[c].y - world.y)) < W(.005)) duplicate = true;
          if (duplicate) continue;
          best = k;
          lowest = z;
        }
        if (best < 0) break;
        V3<R> bestLocal = point(s, b, best);
        V3<R> bestWorld = b.x + rotate(b.q, bestLocal);
        Contact<R> c{};
        c.body = s.body;
        c.shape = int(si);
        c.feature = best;
        c.local = bestLocal;
        c.anchor = {bestWorld.x, bestWorld.y, R(0)};
        c.friction = s.friction;
        for (int d = 0; d < 3; ++d) c.penalty[d] = R(1000);
        for (auto &cached : previous)
          if (cached.other < 0 && cached.shape == int(si) && cached.feature == best) {
            for (int d = 0; d < 3; ++d) { c.lambda[d] = cached.lambda[d]; c.penalty[d] = cached.penalty[d]; }
            if (cached.stick) { c.local = cached.local; c.anchor = cached.anchor; }
            break;
          }
        c.c0 = rmin((b.x + rotate(b.q, c.local)).z, R(0));
        for (int d = 0; d < 3; ++d) {
          c.lambda[d] *= options.alpha * options.gamma;
          c.penalty[d] = rclamp(c.penalty[d] * options.gamma, R(1000), R(1e9));
        }
        if (int(contacts.size()) >= model->contactCapacity) failed = 1;
        else contacts.push_back(c);
        chosen[n++] = bestWorld;
      }
    }
    for (const auto &pair : model->pairs) {
      const auto &sa = model->shapes[pair.a];
      const auto &sb = model->shapes[pair.b];
      const auto &a = bodies[sa.body];
      const auto &b = bodies[sb.body];
      if (a.mass == R(0) && b.mass == R(0)) continue;
      R skin = R(.003) + dt * (norm<R, W>(a.v - b.v) + norm<R, W>(a.w) * sa.boundingRadius +
                               norm<R, W>(b.w) * sb.boundingRadius);
      if (norm<R, W>(a.x - b.x) > sa.boundingRadius + sb.boundingRadius + skin) continue;
      auto hit = convexContact<R, W>(Minkowski<R, W>{sa, sb, a, b, model->points.data(), skin},
                                     rmax(R(1e-8), options.tolerance * R(.1)));
      if (hit.status < 0) { failed = 1; continue; }
      if (hit.status == 0) continue;
      Contact<R> c{};
      c.body = sa.body;
      c.other = sb.body;
      c.shape = pair.a;
      c.otherShape = pair.b;
      c.normal = hit.normal;
      c.tangent1 = unit<R, W>(cross(m_abs(c.normal.x) < R(.8) ? V3<R>{R(1), R(0), R(0)} : V3<R>{R(0), R(1), R(0)}, c.normal));
      c.tangent2 = cross(c.normal, c.tangent1);
      R gap = skin - hit.depth;
      c.local = rotate(conj(a.q), hit.position + scaled(c.normal, gap / R(2)) - a.x);
      c.localB = rotate(conj(b.q), hit.position - scaled(c.normal, gap / R(2)) - b.x);
      c.c0 = rmin(gap, R(0));
      c.friction = pair.friction;
      for (int d = 0; d < 3; ++d) c.penalty[d] = R(1000);
      for (const auto &old : previous)
        if (old.shape == c.shape && old.otherShape == c.otherShape && dot(old.normal, c.normal) > R(.95) &&
            norm<R, W>(rotate(a.q, old.local - c.local)) < R(.005) &&
            norm<R, W>(rotate(b.q, old.localB - c.localB)) < R(.005)) {
          V3<R> f = contactWorld(old, {old.lambda[0], old.lambda[1], old.lambda[2]});
          c.lambda[0] = dot(f, c.tangent1);
          c.lambda[1] = dot(f, c.tangent2);
          c.lambda[2] = dot(f, c.normal);
          for (int d = 0; d < 3; ++d) c.penalty[d] = old.penalty[d];
          break;
        }
      for (int k = 0; k < 3; ++k) {
        c.lambda[k] *= options.alpha * options.gamma;
        c.penalty[k] = rclamp(c.penalty[k] * options.gamma, R(1000), R(1e9));
      }
      if (int(contacts.size()) >= model->contactCapacity) { failed = 1; continue; }
      contacts.push_back(c);
      if (a.mass > R(0) && b.mass > R(0) && colors[c.body] == colors[c.other]) colors[c.other] = colorCount++;
    }
  }
  // Primal block update of one body (kernel.cuh:828-936).
  R updateBody(int bi) {
    const R h = options.dt;
    auto &b = bodies[bi];
    if (b.mass == R(0)) return R(0);
    M6<R> H{};
    V6<R> g{};
    V3<R> dx = b.x - b.xp, theta = qlog<R, W>(qmul(b.q, conj(b.qp)));
    for (int k = 0; k < 3; ++k) {
      H[k][k] = b.mass / (h * h);
      g[k] = H[k][k] * dx[k];
    }
    R a = norm<R, W>(theta);
    // SO(3) log-Jacobian coefficient, formed in double by the reference.
    R coef = W(a) < W(1e-5) ? R(W(1.0) / W(12) + W(a * a / R(720)))
                            : R((W(1) - W(0.5) * W(a) / m_tan(W(0.5) * W(a))) / W(a * a));
    V3<R> rotJ[3];
    for (int k = 0; k < 3; ++k) {
      V3<R> e{};
      e[k] = R(1);
      rotJ[k] = e - scaled(cross(theta, e), R(0.5)) + scaled(cross(theta, cross(theta, e)), coef);
    }
    for (int k = 0; k < 3; ++k) {
      g[k + 3] = dot(rotJ[k], inertiaMul(b, theta)) / (h * h);
      for (int l = 0; l < 3; ++l) H[k + 3][l + 3] = dot(rotJ[k], inertiaMul(b, rotJ[l])) / (h * h);
    }
    for (int adj = model->csrOffsets[bi]; adj < model->csrOffsets[bi + 1]; ++adj) {
      const int ji = model->csrJoints[adj];
      auto &j = joints[ji];
      R C[7]{};
      V6<R> J[7]{};
      const bool parent = bi == j.a;
      const R jointAngle = evaluateJoint(j, C, J, parent ? 0 : 1);
      for (int k = 0; k < (j.limited ? 7 : 5); ++k) {
        R c = C[k] - options.alpha * (k < 5 ? j.c0[k] : rmin(j.c0[k], R(0)));
        R f = j.lambda[k] + j.penalty[k] * c;
        if (k >= 5) f = rmin(f, R(0));
        if (k < 5 || f < R(0)) {
          stamp(H, g, J[k], f, j.penalty[k]);
          if (k < 3) {
            V3<R> e{};
            e[k] = f;
            geometric(H, rotate(b.q, parent ? j.ra : -j.rb), e);
          } else if (k < 5) {
            V3<R> aa = rotate(bodies[j.a].q, j.axisA), ta = rotate(bodies[j.a].q, j.tangentA);
            if (k == 4) ta = cross(aa, ta);
            V3<R> ab = rotate(bodies[j.b].q, j.axisB);
            geometric(H, parent ? ta : ab, scaled(parent ? ab : ta, f));
          }
        }
      }
      R drive = j.kp * wrap<R, W>(jointAngle - j.target) - j.torque;
      R driveStiffness = j.kp;
      if (j.maxTorque > R(0)) {
        if (m_abs(drive) >= j.maxTorque) driveStiffness = R(0);
        drive = rclamp(drive, -j.maxTorque, j.maxTorque);
      }
      stamp(H, g, J[5], drive, driveStiffness);
      R delta = wrap<R, W>(jointAngle - j.angle0), stiff = j.damping / h + j.armature / (h * h),
        force = j.damping / h * delta + j.armature / (h * h) * (delta - h * j.velocity0);
      if (stiff > R(0)) stamp(H, g, J[5], force, stiff);
      if (j.frictionloss > R(0)) {
        R trial = j.lambdaF + j.penaltyF * delta;
        stamp(H, g, J[5], rclamp(trial, -j.frictionloss, j.frictionloss),
              m_abs(trial) < j.frictionloss ? j.penaltyF : R(0));
      }
    }
    for (auto &c : contacts)
      if (c.body == bi || c.other == bi) {
        V3<R> C;
        V6<R> J[3]{};
        contactValues(c, C, J, bi);
        V3<R> f = contactForce(C, c);
        if (f.z < R(0)) {
          for (int k = 0; k < 3; ++k) stamp(H, g, J[k], f[k], c.penalty[k]);
          geometric(H, rotate(b.q, bi == c.body ? c.local : c.localB),
                    scaled(contactWorld(c, f), bi == c.body ? R(1) : R(-1)));
        }
      }
    auto st = solve6(H, g);
    V3<R> tx{st[0], st[1], st[2]}, rx{st[3], st[4], st[5]};
    R scale = rmin(R(1), rmin(R(.1) / rmax(norm<R, W>(tx), R(1e-30)), R(.25) / rmax(norm<R, W>(rx), R(1e-30))));
    b.x = b.x + scaled(tx, scale);
    b.q = qnormalized<R, W>(qmul(qexp<R, W>(scaled(rx, scale)), b.q));
    return rmax(norm<R, W>(tx), norm<R, W>(rx)) * scale;
  }
  // One physics substep (kernel.cuh:937-1095).
  void step() {
    const R h = options.dt;
    if (!(h > R(0)) || options.iterations < 1 || options.alpha < R(0) || options.alpha >= R(1) ||
        options.gamma <= R(0) || options.gamma >= R(1)) {
      failed = 1;
      return;
    }
    diagnostics = {};
    detectContacts();
    if (failed) return;
    for (auto &j : joints) {
      V6<R> A[7];
      evaluateJoint(j, j.c0, A, 2);
      j.angle0 = angle(j);
      j.lambdaF *= options.alpha * options.gamma;
      j.penaltyF = rclamp(j.penaltyF * options.gamma, R(1.0), R(1e7));
      V3<R> axis = rotate(bodies[j.a].q, j.axisA);
      j.velocity0 = dot(bodies[j.b].w - bodies[j.a].w, axis);
      for (int k = 0; k < 7; ++k) {
        j.lambda[k] *= options.alpha * options.gamma;
        j.penalty[k] = rclamp(j.penalty[k] * options.gamma, minimumPenalty<R>(k), maximumPenalty<R>(k));
      }
    }
    for (auto &b : bodies) {
      b.x0 = b.x;
      b.q0 = b.q;
      if (b.mass == R(0)) continue;
      b.xp = b.x + scaled(b.v, h) + scaled(options.gravity + divided(b.force, b.mass), h * h);
      V3<R> wp = b.w + scaled(inertiaMul(b, -cross(b.w, inertiaMul(b, b.w)), true), h);
      b.qp = qmul(qexp<R, W>(scaled(wp, h)), b.q);
      b.x = b.xp;
      b.q = b.qp;
    }
    for (int it = 0; it < options.iterations; ++it) {
      R maxUpdate = R(0);
      for (int color = 0; color < colorCount; ++color)
        for (size_t bi = 0; bi < bodies.size(); ++bi)
          if (colors[bi] == color) maxUpdate = rmax(maxUpdate, updateBody(int(bi)));
      R error = R(0);
      for (auto &j : joints) {
        R C[7]{};
        const R jointAngle = evaluateJoint(j, C, nullptr, 2);
        for (int k = 0; k < (j.limited ? 7 : 5); ++k) {
          R c = C[k] - options.alpha * (k < 5 ? j.c0[k] : rmin(j.c0[k], R(0)));
          R f = j.lambda[k] + j.penalty[k] * c;
          j.lambda[k] = k >= 5 ? rmin(f, R(0)) : f;
          if (k < 5 || f < R(0))
            j.penalty[k] = rmin(j.penalty[k] + (k < 3 ? options.betaLinear : options.betaAngular) * m_abs(c),
                                maximumPenalty<R>(k));
          error = rmax(error, k < 5 ? m_abs(c) : rmax(R(0), -c));
        }
        if (j.frictionloss > R(0)) {
          R delta = wrap<R, W>(jointAngle - j.angle0);
          R trial = j.lambdaF + j.penaltyF * delta;
          j.lambdaF = rclamp(trial, -j.frictionloss, j.frictionloss);
          if (m_abs(trial) < j.frictionloss)
            j.penaltyF = rmin(j.penaltyF + options.betaAngular * m_abs(delta), R(1e7));
          R residualTrial = j.lambdaF + j.penaltyF * wrap<R, W>(jointAngle - j.angle0);
          error = rmax(error, m_abs(j.lambdaF - rclamp(residualTrial, -j.frictionloss, j.frictionloss)) / j.penaltyF);
        }
      }
      for (auto &c : contacts) {
        V3<R> C;
        V6<R> J[3]{};
        contactValues(c, C, J);
        V3<R> f = contactForce(C, c);
        R trial = m_hypot(c.lambda[0] + c.penalty[0] * C.x, c.lambda[1] + c.penalty[1] * C.y);
        c.stick = trial <= -c.friction * f.z && W(m_hypot(C.x, C.y)) < W(1e-5);
        for (int k = 0; k < 3; ++k) {
          c.lambda[k] = f[k];
          if (f.z < R(0) && (k == 2 || trial <= -c.friction * f.z))
            c.penalty[k] = rmin(c.penalty[k] + options.betaLinear * m_abs(C[k]), R(1e9));
        }
      }
      for (auto &c : contacts) {
        V3<R> C;
        V6<R> J[3]{};
        contactValues(c, C, J);
        error = rmax(error, rmax(R(0), -C.z));
      }
      diagnostics.update = maxUpdate;
      diagnostics.iterations = it + 1;
      diagnostics.converged = maxUpdate < options.tolerance && error < options.tolerance;
      if (diagnostics.converged) break;
    }
    for (auto &b : bodies)
      if (b.mass > R(0)) {
        b.v = divided(b.x - b.x0, h);
        b.w = divided(qlog<R, W>(qmul(b.q, conj(b.q0))), h);
        if (!m_finite(norm<R, W>(b.x) + norm<R, W>(b.v) + norm<R, W>(b.w))) {
          failed = 1;
          return;
        }
      }
    for (auto &j : joints) {
      R C[7]{};
      evaluateJoint(j, C, nullptr, 2);
      for (int k = 0; k < 3; ++k) diagnostics.jointError = rmax(diagnostics.jointError, m_abs(C[k]));
      for (int k = 3; k < 5; ++k) diagnostics.axisError = rmax(diagnostics.axisError, m_abs(C[k]));
    }
    for (auto &c : contacts) {
      V3<R> C;
      V6<R> J[3];
      contactValues(c, C, J);
      diagnostics.penetration = rmax(diagnostics.penetration, rmax(R(0), -(C.z + options.alpha * c.c0)));
    }
    diagnostics.contacts = int(contacts.size());
  }
  // RNEA at zero generalized acceleration (kernel.cuh:504-554).
  template <class T> void generalizedLoads(V3<R> rootOffset, T *out) const {
    const size_t nb = bodies.size();
    std::vector<V3<R>> acc(nb), alpha(nb), force(nb), moment(nb), contact(nb), contactMoment(nb);
    const auto &root = bodies[1];
    acc[1] = cross(root.w, cross(root.w, rotate(root.q, rootOffset)));
    for (auto &j : joints) {
      const auto &a = bodies[j.a];
      const auto &b = bodies[j.b];
      V3<R> axis = rotate(a.q, j.axisA), ra = rotate(a.q, j.ra), rb = rotate(b.q, j.rb);
      R speed = dot(b.w - a.w, axis);
      alpha[j.b] = alpha[j.a] + scaled(cross(a.w, axis), speed);
      acc[j.b] = acc[j.a] + cross(alpha[j.a], ra) + cross(a.w, cross(a.w, ra)) - cross(alpha[j.b], rb) -
                 cross(b.w, cross(b.w, rb));
    }
    for (size_t i = 1; i < nb; ++i) {
      auto b = bodies[i];
      b.q0 = b.q;
      force[i] = scaled(acc[i] - options.gravity, b.mass);
      moment[i] = inertiaMul(b, alpha[i]) + cross(b.w, inertiaMul(b, b.w));
    }
    for (auto &c : contacts) {
      V3<R> f = -contactWorld(c, {c.lambda[0], c.lambda[1], c.lambda[2]});
      contact[c.body] = contact[c.body] + f;
      contactMoment[c.body] = contactMoment[c.body] + cross(rotate(bodies[c.body].q, c.local), f);
      if (c.other >= 0) {
        contact[c.other] = contact[c.other] + (-f);
        contactMoment[c.other] = contactMoment[c.other] + cross(rotate(bodies[c.other].q, c.localB), -f);
      }
    }
    for (int k = int(joints.size()) - 1; k >= 0; --k) {
      const auto &j = joints[k];
      const auto &a = bodies[j.a];
      const auto &b = bodies[j.b];
      V3<R> axis = rotate(a.q, j.axisA), rb = rotate(b.q, j.rb), shift = b.x - a.x;
      R o0 = dot(axis, moment[j.b] - cross(rb, force[j.b]));
      R o1 = dot(axis, contactMoment[j.b] - cross(rb, contact[j.b])) +
             (j.limited ? -j.lambda[5] + j.lambda[6] : R(0));
      R motor = j.torque - j.kp * wrap<R, W>(angle(j) - j.target);
      R o2 = j.maxTorque > R(0) ? rclamp(motor, -j.maxTorque, j.maxTorque) : motor;
      out[3 * k] = T(raw(o0));
      out[3 * k + 1] = T(raw(o1));
      out[3 * k + 2] = T(raw(o2));
      moment[j.a] = moment[j.a] + (moment[j.b] + cross(shift, force[j.b]));
      force[j.a] = force[j.a] + force[j.b];
      contactMoment[j.a] = contactMoment[j.a] + (contactMoment[j.b] + cross(shift, contact[j.b]));
      contact[j.a] = contact[j.a] + contact[j.b];
    }
  }
  template <class T> void snapshot(T *b, T *j, T *d) const {   // kernel.cuh:555-575
    for (size_t i = 0; i < bodies.size(); ++i) {
      auto &v = bodies[i];
      R row[] = {v.x.x, v.x.y, v.x.z, v.q.w, v.q.x, v.q.y, v.q.z, v.v.x, v.v.y, v.v.z, v.w.x, v.w.y, v.w.z};
      for (int k = 0; k < 13; ++k) b[13 * i + k] = T(raw(row[k]));
    }
    for (size_t i = 0; i < joints.size(); ++i) {
      auto &v = joints[i];
      j[2 * i] = T(raw(angle(v)));
      j[2 * i + 1] = T(raw(dot(bodies[v.b].w - bodies[v.a].w, rotate(bodies[v.a].q, v.axisA))));
    }
    d[0] = T(raw(diagnostics.jointError));
    d[1] = T(raw(diagnostics.penetration));
    d[2] = T(diagnostics.contacts);
    d[3] = T(diagnostics.converged);
    d[4] = T(raw(diagnostics.axisError));
    d[5] = T(failed);
  }
};

}  // namespace avbd_oracle
