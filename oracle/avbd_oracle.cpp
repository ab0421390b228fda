// C-ABI over the CPU restatement in avbd_oracle.hpp -- TEST INFRASTRUCTURE
// ONLY (the checker for tests/, __graft_entry__.smoke() and bench.py's
// cpu_baseline leg; never linked into the product).
//
// The batch mirrors the reference CPU twin _duck_reference.CpuBatch32/64
// (src/cuda/cpu_bindings.cpp:20-168): env-strided worker threads, numpy-style
// dense arrays in and out.  step() can follow either the CPU twin's input
// handling (cpu_bindings.cpp:69-112) or the CUDA kernel's
// (src/cuda/extension.cu:78-114), which differ only for envs given non-finite
// controls.
//
// Portable per-env record (shared with the product library's export/import
// entry points, all values in the batch scalar type):
//   [0] failed [1] contact count [2] jointError [3] penetration [4] contacts
//   [5] converged [6] axisError [7] iterations
//   bodies   B x 16 : x(3) q(4) v(3) w(3) force(3)
//   joints   J x 22 : lambda(7) penalty(7) lambdaF penaltyF target kp
//                     maxTorque torque frictionloss damping
//   contacts C x 32 : body shape feature other otherShape stick local(3)
//                     anchor(3) localB(3) tangent1(3) tangent2(3) normal(3)
//                     friction c0 lambda(3) penalty(3)
// with C = contact bound of the model (pairs + 4 per ground shape).
#include "avbd_oracle.hpp"

#include <cstring>
#include <memory>
#include <mutex>
#include <thread>

using namespace avbd_oracle;

namespace {
thread_local std::string lastError;

int contactBound(const DModel &m) {
  int bound = int(m.pairs.size());
  if (m.ground)
    for (const auto &s : m.shapes)
      if (s.ground && m.bodies[s.body].mass > 0) bound += 4;
  return bound;
}

struct BatchBase {
  virtual ~BatchBase() = default;
  int n = 0, bodies = 0, joints = 0, bound = 0, fp64 = 0;
  virtual void reset(const uint8_t *mask, const void *q, const void *roots) = 0;
  virtual void step(const void *target, const void *forces, int substeps, double kp, double limit,
                    int threads, int cudaSemantics) = 0;
  virtual void stepMotor(const void *motor, const void *forces, int threads) = 0;
  virtual void state(void *b, void *j, void *d) = 0;
  virtual void contactForces(void *out, bool groundOnly) = 0;
  virtual void selfContactStats(void *out) = 0;
  virtual void contactCounts(void *out) = 0;
  virtual void generalizedLoads(const void *offset, void *out) = 0;
  virtual int contacts(int env, int32_t *keys, int capacity) = 0;
  virtual void exportEnv(int env, void *dst) = 0;
  virtual void importEnv(int env, const void *src) = 0;
  virtual int colorCount(int env) = 0;
  int recordLength() const { return 8 + bodies * 16 + joints * 22 + bound * 32; }
};

template <class F> void parallel(int n, int threads, F &&work) {
  int workers = std::max(1, std::min(n, threads));
  std::vector<std::thread> pool;
  for (int w = 1; w < workers; ++w)
    pool.emplace_back([&, w] { for (int e = w; e < n; e += workers) work(e); });
  for (int e = 0; e < n; e += workers) work(e);
  for (auto &t : pool) t.join();
}

// Loads one portable record (the layout exportEnv writes) into an env of any
// scalar type: the oracle batch's own, or the counting scalar's.
template <class S, class Src> void loadRecord(S &s, const Src *o, int bodies, int joints, int bound) {
  using Item = typename std::decay_t<decltype(s.contacts)>::value_type;
  s.failed = int(o[0]);
  int count = int(o[1]);
  if (count < 0 || count > bound) throw std::invalid_argument("contact count out of range");
  s.diagnostics = {};
  s.diagnostics.jointError = o[2];
  s.diagnostics.penetration = o[3];
  s.diagnostics.contacts = int(o[4]);
  s.diagnostics.converged = o[5] != Src(0);
  s.diagnostics.axisError = o[6];
  s.diagnostics.iterations = int(o[7]);
  const Src *b = o + 8;
  for (int i = 0; i < bodies; ++i, b += 16) {
    auto &v = s.bodies[i];
    v.x = {b[0], b[1], b[2]};
    v.q = {b[3], b[4], b[5], b[6]};
    v.v = {b[7], b[8], b[9]};
    v.w = {b[10], b[11], b[12]};
    v.force = {b[13], b[14], b[15]};
  }
  const Src *j = o + 8 + bodies * 16;
  for (int i = 0; i < joints; ++i, j += 22) {
    auto &v = s.joints[i];
    for (int k = 0; k < 7; ++k) { v.lambda[k] = j[k]; v.penalty[k] = j[7 + k]; }
    v.lambdaF = j[14]; v.penaltyF = j[15]; v.target = j[16]; v.kp = j[17];
    v.maxTorque = j[18]; v.torque = j[19]; v.frictionloss = j[20]; v.damping = j[21];
  }
  const Src *c = o + 8 + bodies * 16 + joints * 22;
  s.contacts.assign(count, Item{});
  for (int i = 0; i < count; ++i, c += 32) {
    auto &v = s.contacts[i];
    v.body = int(c[0]); v.shape = int(c[1]); v.feature = int(c[2]); v.other = int(c[3]);
    v.otherShape = int(c[4]); v.stick = c[5] != Src(0);
    v.local = {c[6], c[7], c[8]}; v.anchor = {c[9], c[10], c[11]}; v.localB = {c[12], c[13], c[14]};
    v.tangent1 = {c[15], c[16], c[17]}; v.tangent2 = {c[18], c[19], c[20]}; v.normal = {c[21], c[22], c[23]};
    v.friction = c[24]; v.c0 = c[25];
    for (int k = 0; k < 3; ++k) { v.lambda[k] = c[26 + k]; v.penalty[k] = c[29 + k]; }
  }
}

template <class R> struct Batch final : BatchBase {
  Model<R> model;
  std::vector<Env<R, double>> envs;
  Batch(const DModel &d, int count, double dt, int iterations, int capacity, int maxPairs = 32) {
    model = convertModel<R>(d, dt, iterations, capacity, 32, 32, maxPairs);
    n = count;
    bodies = int(model.bodies.size());
    joints = int(model.joints.size());
    bound = contactBound(d);
    fp64 = std::is_same_v<R, double>;
    envs.resize(count);
    for (auto &e : envs) e.initialize(&model);
  }
  void reset(const uint8_t *mask, const void *qv, const void *rv) override {
    const R *q = static_cast<const R *>(qv), *roots = static_cast<const R *>(rv);
    for (int e = 0; e < n; ++e) {
      if (!mask[e]) continue;
      bool valid = true;
      for (int j = 0; j < joints; ++j) valid &= std::isfinite(q[e * joints + j]);
      for (int k = 0; k < 6; ++k) valid &= std::isfinite(roots[e * 6 + k]);
      if (!valid) { envs[e].failed = 1; continue; }
      envs[e].initialize(&model);
      envs[e].resetPose(q + e * joints, roots + e * 6);
    }
  }
  void step(const void *tv, const void *fv, int substeps, double kp, double limit, int threads,
            int cudaSemantics) override {
    const R *targets = static_cast<const R *>(tv), *external = static_cast<const R *>(fv);
    parallel(n, threads, [&](int e) {
      auto &s = envs[e];
      if (cudaSemantics) {
        for (int j = 0; j < joints; ++j)
          if (!std::isfinite(targets[e * joints + j])) s.failed = 1;
        for (int k = 0; k < 3; ++k)
          if (!std::isfinite(external[e * 3 + k])) s.failed = 1;
        if (s.failed) return;
      }
      for (int j = 0; j < joints; ++j) {
        R t = targets[e * joints + j];
        if (!std::isfinite(t)) s.failed = 1;
        s.joints[j].target = t;
        s.joints[j].kp = R(kp);
        s.joints[j].maxTorque = R(limit);
        s.joints[j].torque = model.joints[j].torque;
        s.joints[j].frictionloss = model.joints[j].frictionloss;
        s.joints[j].damping = model.joints[j].damping;
      }
      for (int k = 0; k < 3; ++k)
        if (!std::isfinite(external[e * 3 + k])) s.failed = 1;
      if (s.failed) return;
      s.bodies[1].force = {external[e * 3], external[e * 3 + 1], external[e * 3 + 2]};
      s.advance(substeps);
    });
  }
  void stepMotor(const void *mv, const void *fv, int threads) override {
    const R *motor = static_cast<const R *>(mv), *forces = static_cast<const R *>(fv);
    parallel(n, threads, [&](int e) {
      auto &s = envs[e];
      s.setMotor(motor + e * joints * 3, forces + e * 3);
      if (!s.failed) s.advance(1);
    });
  }
  void state(void *bv, void *jv, void *dv) override {
    R *b = static_cast<R *>(bv), *j = static_cast<R *>(jv), *d = static_cast<R *>(dv);
    for (int e = 0; e < n; ++e) envs[e].snapshot(b + e * bodies * 13, j + e * joints * 2, d + e * 6);
  }
  void contactForces(void *out, bool groundOnly) override {
    for (int e = 0; e < n; ++e) envs[e].contactForces(static_cast<R *>(out) + e * bodies * 3, groundOnly);
  }
  void selfContactStats(void *out) override {
    for (int e = 0; e < n; ++e) envs[e].selfContactStats(static_cast<R *>(out) + 2 * e);
  }
  void contactCounts(void *out) override {
    for (int e = 0; e < n; ++e) envs[e].contactCounts(static_cast<R *>(out) + 2 * e);
  }
  void generalizedLoads(const void *ov, void *out) override {
    const R *p = static_cast<const R *>(ov);
    for (int e = 0; e < n; ++e) {
      for (int k = 0; k < 3; ++k)
        if (!std::isfinite(p[3 * e + k])) throw std::invalid_argument("Invalid root COM offset");
      envs[e].generalizedLoads(V3<R>{p[3 * e], p[3 * e + 1], p[3 * e + 2]},
                               static_cast<R *>(out) + e * joints * 3);
    }
  }
  int contacts(int env, int32_t *keys, int capacity) override {
    const auto &list = envs.at(env).contacts;
    int count = int(list.size());
    for (int i = 0; i < std::min(count, capacity); ++i) {
      const auto &c = list[i];
      int32_t row[5] = {c.body, c.shape, c.feature, c.other, c.otherShape};
      std::memcpy(keys + 5 * i, row, sizeof(row));
    }
    return count;
  }
  int colorCount(int env) override { return envs.at(env).colorCount; }
  void exportEnv(int env, void *dst) override {
    const auto &s = envs.at(env);
    R *o = static_cast<R *>(dst);
    std::fill(o, o + recordLength(), R(0));
    o[0] = R(s.failed);
    o[1] = R(s.contacts.size());
    o[2] = s.diagnostics.jointError;
    o[3] = s.diagnostics.penetration;
    o[4] = R(s.diagnostics.contacts);
    o[5] = R(s.diagnostics.converged);
    o[6] = s.diagnostics.axisError;
    o[7] = R(s.diagnostics.iterations);
    R *b = o + 8;
    for (int i = 0; i < bodies; ++i, b += 16) {
      const auto &v = s.bodies[i];
      R row[16] = {v.x.x, v.x.y, v.x.z, v.q.w, v.q.x, v.q.y, v.q.z, v.v.x, v.v.y, v.v.z,
                   v.w.x, v.w.y, v.w.z, v.force.x, v.force.y, v.force.z};
      std::copy(row, row + 16, b);
    }
    R *j = o + 8 + bodies * 16;
    for (int i = 0; i < joints; ++i, j += 22) {
      const auto &v = s.joints[i];
      for (int k = 0; k < 7; ++k) { j[k] = v.lambda[k]; j[7 + k] = v.penalty[k]; }
      R tail[8] = {v.lambdaF, v.penaltyF, v.target, v.kp, v.maxTorque, v.torque, v.frictionloss, v.damping};
      std::copy(tail, tail + 8, j + 14);
    }
    R *c = o + 8 + bodies * 16 + joints * 22;
    for (size_t i = 0; i < s.contacts.size() && int(i) < bound; ++i, c += 32) {
      const auto &v = s.contacts[i];
      R row[32] = {R(v.body), R(v.shape), R(v.feature), R(v.other), R(v.otherShape), R(v.stick),
                   v.local.x, v.local.y, v.local.z, v.anchor.x, v.anchor.y, v.anchor.z,
                   v.localB.x, v.localB.y, v.localB.z, v.tangent1.x, v.tangent1.y, v.tangent1.z,
                   v.tangent2.x, v.tangent2.y, v.tangent2.z, v.normal.x, v.normal.y, v.normal.z,
                   v.friction, v.c0, v.lambda[0], v.lambda[1], v.lambda[2],
                   v.penalty[0], v.penalty[1], v.penalty[2]};
      std::copy(row, row + 32, c);
    }
  }
  void importEnv(int env, const void *src) override {
    loadRecord(envs.at(env), static_cast<const R *>(src), bodies, joints, bound);
  }
};

template <class F> int guarded(F &&f) {
  try {
    f();
    return 0;
  } catch (const std::exception &e) {
    lastError = e.what();
    return 1;
  }
}
BatchBase *B(void *p) { return static_cast<BatchBase *>(p); }
}  // namespace

extern "C" {
const char *avbd_oracle_last_error() { return lastError.c_str(); }

void *avbd_oracle_create_ex(const char *path, int n, double dt, int iterations, int fp64, int capacity,
                            int maxPairs) {
  try {
    if (!(n > 0 && n <= 65536 && dt > 0 && std::isfinite(dt) && iterations > 0 && maxPairs >= 0 && maxPairs <= 128))
      throw std::invalid_argument("Invalid batch parameters");
    DModel d = loadDuck(path, maxPairs);
    if (fp64) return new Batch<double>(d, n, dt, iterations, capacity, maxPairs);
    return new Batch<float>(d, n, dt, iterations, capacity, maxPairs);
  } catch (const std::exception &e) {
    lastError = e.what();
    return nullptr;
  }
}
void *avbd_oracle_create(const char *path, int n, double dt, int iterations, int fp64, int capacity) {
  return avbd_oracle_create_ex(path, n, dt, iterations, fp64, capacity, 32);
}
void avbd_oracle_destroy(void *b) { delete B(b); }
int avbd_oracle_info(void *b, int32_t *out) {
  out[0] = B(b)->n; out[1] = B(b)->bodies; out[2] = B(b)->joints; out[3] = B(b)->bound;
  out[4] = B(b)->recordLength(); out[5] = B(b)->fp64;
  return 0;
}
int avbd_oracle_reset(void *b, const uint8_t *mask, const void *q, const void *roots) {
  return guarded([&] { B(b)->reset(mask, q, roots); });
}
int avbd_oracle_step(void *b, const void *target, const void *forces, int substeps, double kp,
                     double limit, int threads, int cudaSemantics) {
  return guarded([&] {
    if (!(substeps > 0 && kp >= 0 && std::isfinite(kp) && limit >= 0 && std::isfinite(limit)))
      throw std::invalid_argument("Invalid controls");
    B(b)->step(target, forces, substeps, kp, limit, threads, cudaSemantics);
  });
}
int avbd_oracle_step_motor(void *b, const void *motor, const void *forces, int threads) {
  return guarded([&] { B(b)->stepMotor(motor, forces, threads); });
}
int avbd_oracle_state(void *b, void *bodies, void *joints, void *diag) {
  return guarded([&] { B(b)->state(bodies, joints, diag); });
}
int avbd_oracle_contact_forces(void *b, void *out, int groundOnly) {
  return guarded([&] { B(b)->contactForces(out, groundOnly != 0); });
}
int avbd_oracle_self_contact_stats(void *b, void *out) {
  return guarded([&] { B(b)->selfContactStats(out); });
}
int avbd_oracle_contact_counts(void *b, void *out) {
  return guarded([&] { B(b)->contactCounts(out); });
}
int avbd_oracle_generalized_loads(void *b, const void *offset, void *out) {
  return guarded([&] { B(b)->generalizedLoads(offset, out); });
}
int avbd_oracle_contacts(void *b, int env, int32_t *keys, int capacity) {
  int count = -1;
  if (guarded([&] { count = B(b)->contacts(env, keys, capacity); })) return -1;
  return count;
}
int avbd_oracle_color_count(void *b, int env) { return B(b)->colorCount(env); }
int avbd_oracle_export(void *b, int env, void *dst) {
  return guarded([&] { B(b)->exportEnv(env, dst); });
}
int avbd_oracle_import(void *b, int env, const void *src) {
  return guarded([&] { B(b)->importEnv(env, src); });
}

// Counts the algorithmic floating-point operations of `steps` control steps
// of the fp32 solver on n envs: targets [steps][n][J] and forces [n][3] are
// float32.  The run starts from `records` ([n][record length] float32
// portable records, e.g. states exported from a GPU batch) when given, else
// from a reset to q = home, roots = 0.  out[0..9] receives
// add, mul, div, sqrt, sin, cos, tan, atan2, hypot, remainder counts; out[10]
// the number of GS iterations actually executed, out[11] the physics steps.
// A failed env stops advancing (its remaining steps still count in out[11]).
int avbd_oracle_count_ops(const char *path, int n, double dt, int iterations, const float *home,
                          const float *records, const float *targets, const float *forces, int steps,
                          int substeps, double kp, double limit, int threads, uint64_t *out) {
  return guarded([&] {
    using T = Tally<float>;
    DModel d = loadDuck(path);
    Model<T> model = convertModel<T>(d, dt, iterations, 160);
    const int nj = int(model.joints.size());
    std::vector<Env<T, Tally<double>>> envs(n);
    std::vector<float> roots(6, 0.f);
    const int nb = int(model.bodies.size()), bound = contactBound(d);
    const int length = 8 + 16 * nb + 22 * nj + 32 * bound;
    for (int e = 0; e < n; ++e) {
      envs[e].initialize(&model);
      if (records) loadRecord(envs[e], records + size_t(e) * length, nb, nj, bound);
      else envs[e].resetPose(home, roots.data());
    }
    // Envs are independent: `threads` workers take every threads-th env and
    // run all its steps; each worker's thread-local tally is summed at the end.
    OpCounts total{};
    uint64_t iters = 0;
    std::mutex sum;
    auto work = [&](int w, int workers) {
      counts() = {};
      uint64_t mine = 0;
      for (int e = w; e < n; e += workers) {
        auto &env = envs[e];
        for (int s = 0; s < steps && !env.failed; ++s) {
          for (int j = 0; j < nj; ++j) {
            env.joints[j].target = targets[(size_t(s) * n + e) * nj + j];
            env.joints[j].kp = T(float(kp));
            env.joints[j].maxTorque = T(float(limit));
            env.joints[j].torque = model.joints[j].torque;
            env.joints[j].frictionloss = model.joints[j].frictionloss;
            env.joints[j].damping = model.joints[j].damping;
          }
          env.bodies[1].force = {T(forces[3 * e]), T(forces[3 * e + 1]), T(forces[3 * e + 2])};
          env.advance(substeps);
          mine += env.diagnostics.iterations;
        }
      }
      const OpCounts &c = counts();
      std::lock_guard<std::mutex> lock(sum);
      total.add += c.add; total.mul += c.mul; total.div += c.div; total.sqrt += c.sqrt;
      total.sin += c.sin; total.cos += c.cos; total.tan += c.tan; total.atan2 += c.atan2;
      total.hypot += c.hypot; total.rem += c.rem;
      iters += mine;
    };
    const int workers = std::max(1, std::min(n, threads));
    std::vector<std::thread> pool;
    for (int w = 1; w < workers; ++w) pool.emplace_back(work, w, workers);
    work(0, workers);
    for (auto &t : pool) t.join();
    const OpCounts &c = total;
    uint64_t v[12] = {c.add, c.mul, c.div, c.sqrt, c.sin, c.cos, c.tan, c.atan2, c.hypot, c.rem,
                      iters, uint64_t(steps) * n * substeps};
    std::memcpy(out, v, sizeof(v));
  });
}
}
