// C ABI of the B200 AVBD library (declared in include/duck_b200.h).
//
// A duck_batch owns: the flat device model, the convex point pool, and one
// portable record per environment (header, bodies, joints, contacts).  Every
// entry point validates its arguments on the host, orders itself after the
// batch's previous work with a private event (the reference's wait()/record(),
// src/cuda/extension.cu:203-205) and launches on the caller's stream.
#include "../../include/duck_b200.h"
#include "aux_kernels.cuh"
#include "bam_kernels.cuh"
#include "ppo_kernels.cuh"

#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

using namespace duckb200;

namespace {
thread_local std::string lastError;

struct CudaError : std::runtime_error {
  using std::runtime_error::runtime_error;
};
void check(cudaError_t e, const char *what) {
  if (e != cudaSuccess) throw CudaError(std::string(what) + ": " + cudaGetErrorString(e));
}
void require(bool c, const char *msg) {
  if (!c) throw std::invalid_argument(msg);
}
// Lanes per environment: the smallest power of two (>= 4) holding the largest
// colour class, unless DUCK_B200_LANES (4, 8, 16 or 32) asks for a wider team.
int teamSize(int colorMax) {
  int t = 4;
  while (t < colorMax && t < 32) t *= 2;
  if (const char *env = std::getenv("DUCK_B200_LANES")) {
    int want = std::atoi(env);
    if ((want == 4 || want == 8 || want == 16 || want == 32) && want >= t) t = want;
  }
  return t;
}
}  // namespace

struct duck_batch {
  int device = 0, fp64 = 0, n = 0, nb = 0, nj = 0, np = 0, bound = 0, recordLength = 0, recordStride = 0;
  int T = 8, teamsPerBlock = 4, smemPerBlock = 0;
  Layout layout{};
  void *devModel = nullptr, *points = nullptr, *records = nullptr;
  // Per-environment parameters (duck_batch_set_parameters), nullptr = model's.
  void *envMass = nullptr, *envInertia = nullptr, *envFriction = nullptr;
  size_t modelBytes = 0;
  cudaEvent_t ready = nullptr;
  std::vector<std::string> names;
  std::shared_ptr<void> hostModel;  // HostModel<float|double>
  int64_t launches = 0;
};

namespace {

template <class R> const HostModel<R> &host(const duck_batch *b) {
  return *static_cast<const HostModel<R> *>(b->hostModel.get());
}

struct DeviceGuard {
  int previous = 0;
  explicit DeviceGuard(int device) {
    check(cudaGetDevice(&previous), "cudaGetDevice");
    check(cudaSetDevice(device), "cudaSetDevice");
  }
  ~DeviceGuard() { cudaSetDevice(previous); }
};

// Calls are ordered across streams by the batch's private event.  While the
// stream is being captured into a CUDA graph the event is left alone: the
// graph's own edges order the captured work, and an event recorded outside the
// capture cannot be waited on inside it.
bool capturing(cudaStream_t s) {
  cudaStreamCaptureStatus status = cudaStreamCaptureStatusNone;
  check(cudaStreamIsCapturing(s, &status), "cudaStreamIsCapturing");
  return status != cudaStreamCaptureStatusNone;
}
void begin(duck_batch *b, cudaStream_t s) {
  if (!capturing(s)) check(cudaStreamWaitEvent(s, b->ready, 0), "cudaStreamWaitEvent");
}
void finish(duck_batch *b, cudaStream_t s) {
  check(cudaGetLastError(), "kernel launch");
  if (!capturing(s)) check(cudaEventRecord(b->ready, s), "cudaEventRecord");
}
int blocksFor(long long threads, int per) { return int((threads + per - 1) / per); }

// The step kernel instantiation for a batch: its team width, and whether its
// model has body-collision pairs (without them the pair code is compiled out).
template <class R, class F> void withAdvance(const duck_batch *b, F &&f) {
  const bool pairs = b->np > 0;
  switch (b->T) {
    case 4: pairs ? f(advanceKernel<R, 4, true>) : f(advanceKernel<R, 4, false>); break;
    case 8: pairs ? f(advanceKernel<R, 8, true>) : f(advanceKernel<R, 8, false>); break;
    case 16: pairs ? f(advanceKernel<R, 16, true>) : f(advanceKernel<R, 16, false>); break;
    default: pairs ? f(advanceKernel<R, 32, true>) : f(advanceKernel<R, 32, false>); break;
  }
}

template <class R> void setupAdvance(duck_batch *b) {
  withAdvance<R>(b, [&](auto kernel) {
    check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, b->smemPerBlock),
          "cudaFuncSetAttribute");
  });
}

template <class R> void launchAdvance(duck_batch *b, const StepArgs &stepArgs, cudaStream_t s) {
  StepArgs args = stepArgs;
  args.mass = b->envMass;
  args.inertia = b->envInertia;
  args.friction = b->envFriction;
  const int grid = blocksFor(b->n, b->teamsPerBlock);
  const R *pts = static_cast<const R *>(b->points);
  const DevModel<R> *m = static_cast<const DevModel<R> *>(b->devModel);
  R *rec = static_cast<R *>(b->records);
  withAdvance<R>(b, [&](auto kernel) {
    kernel<<<grid, 32, b->smemPerBlock, s>>>(m, pts, rec, b->recordStride, b->n, b->layout, args);
  });
  ++b->launches;
}

template <class R> void launchReset(duck_batch *b, const uint8_t *mask, const void *q, const void *roots, int pose,
                                    cudaStream_t s) {
  resetKernel<R><<<blocksFor(b->n, 128), 128, 0, s>>>(
      static_cast<const DevModel<R> *>(b->devModel), static_cast<R *>(b->records), b->recordStride, b->n, mask,
      static_cast<const R *>(q), static_cast<const R *>(roots), pose);
  ++b->launches;
}

template <class R> duck_batch *create(const ParsedModel &parsed, int n, double dt, int iterations, int device,
                                      bool specialized, int maxPairs, cudaStream_t s) {
  auto hm = std::make_shared<HostModel<R>>(convertModel<R>(parsed, dt, iterations, specialized, maxPairs));
  auto b = std::make_unique<duck_batch>();
  b->device = device;
  b->fp64 = std::is_same_v<R, double>;
  b->n = n;
  b->nb = hm->dev.nb;
  b->nj = hm->dev.nj;
  b->np = hm->dev.np;
  b->bound = hm->dev.bound;
  b->names = hm->jointNames;
  b->recordLength = kRecHeader + kRecBody * b->nb + kRecJoint * b->nj + kRecContact * b->bound;
  b->recordStride = (b->recordLength + 31) & ~31;
  b->layout = makeLayout(hm->dev);
  b->T = teamSize(hm->dev.colorMax);
  scheduleSweep(hm->dev, b->T);
  b->teamsPerBlock = 32 / b->T;
  b->smemPerBlock = int(b->teamsPerBlock * b->layout.size * sizeof(R));
  int maxShared = 0;
  check(cudaDeviceGetAttribute(&maxShared, cudaDevAttrMaxSharedMemoryPerBlockOptin, device), "cudaDeviceGetAttribute");
  require(b->smemPerBlock <= maxShared, "Device shared memory is too small for this model");
  b->hostModel = hm;
  b->modelBytes = sizeof(DevModel<R>);
  check(cudaMalloc(&b->devModel, sizeof(DevModel<R>)), "cudaMalloc model");
  size_t pointBytes = std::max<size_t>(1, hm->points.size()) * sizeof(R);
  check(cudaMalloc(&b->points, pointBytes), "cudaMalloc points");
  check(cudaMalloc(&b->records, size_t(n) * b->recordStride * sizeof(R)), "cudaMalloc records");
  check(cudaMemsetAsync(b->records, 0, size_t(n) * b->recordStride * sizeof(R), s), "cudaMemsetAsync");
  check(cudaMemcpyAsync(b->devModel, &hm->dev, sizeof(DevModel<R>), cudaMemcpyHostToDevice, s), "copy model");
  if (!hm->points.empty())
    check(cudaMemcpyAsync(b->points, hm->points.data(), hm->points.size() * sizeof(R), cudaMemcpyHostToDevice, s),
          "copy points");
  setupAdvance<R>(b.get());
  launchReset<R>(b.get(), nullptr, nullptr, nullptr, 0, s);
  check(cudaGetLastError(), "initialise");
  check(cudaStreamSynchronize(s), "cudaStreamSynchronize");
  check(cudaEventCreateWithFlags(&b->ready, cudaEventDisableTiming), "cudaEventCreate");
  check(cudaEventRecord(b->ready, s), "cudaEventRecord");
  return b.release();
}

template <class F> int guarded(F &&f) {
  try {
    f();
    return DUCK_OK;
  } catch (const std::invalid_argument &e) {
    lastError = e.what();
    return DUCK_EINVAL;
  } catch (const CudaError &e) {
    lastError = e.what();
    return DUCK_ECUDA;
  } catch (const std::exception &e) {
    lastError = e.what();
    return DUCK_EMODEL;
  }
}

}  // namespace

namespace {
template <class R> void snapshot(duck_batch *b, void *bodies, void *joints, void *diag, cudaStream_t s) {
  long long items = (long long)b->n * (b->nb + b->nj + 1);
  snapshotKernel<R><<<blocksFor(items, 256), 256, 0, s>>>(
      static_cast<const DevModel<R> *>(b->devModel), static_cast<const R *>(b->records), b->recordStride, b->n,
      static_cast<R *>(bodies), static_cast<R *>(joints), static_cast<R *>(diag));
  ++b->launches;
}
template <class R> void forcesLaunch(duck_batch *b, void *out, int groundOnly, cudaStream_t s) {
  contactForcesKernel<R><<<blocksFor(b->n, 128), 128, 0, s>>>(
      static_cast<const DevModel<R> *>(b->devModel), static_cast<const R *>(b->records), b->recordStride, b->n,
      static_cast<R *>(out), groundOnly);
  ++b->launches;
}
template <class R> void statsLaunch(duck_batch *b, void *counts, void *self, cudaStream_t s) {
  contactStatsKernel<R><<<blocksFor(b->n, 128), 128, 0, s>>>(
      static_cast<const DevModel<R> *>(b->devModel), static_cast<const R *>(b->records), b->recordStride, b->n,
      static_cast<R *>(counts), static_cast<R *>(self));
  ++b->launches;
}
template <class R> void loadsLaunch(duck_batch *b, const void *offset, void *out, cudaStream_t s) {
  static int limit[2][64] = {};
  const int need = int(18 * b->nb * 32 * sizeof(R));
  int &have = limit[sizeof(R) == 8][b->device & 63];
  if (need > have) {
    check(cudaFuncSetAttribute(generalizedLoadsKernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, need),
          "cudaFuncSetAttribute");
    have = need;
  }
  generalizedLoadsKernel<R><<<blocksFor(b->n, 32), 32, need, s>>>(
      static_cast<const DevModel<R> *>(b->devModel), static_cast<const R *>(b->records), b->recordStride, b->n,
      static_cast<const R *>(offset), static_cast<R *>(out), static_cast<const R *>(b->envMass),
      static_cast<const R *>(b->envInertia));
  ++b->launches;
}
}  // namespace

extern "C" {

const char *duck_last_error(void) { return lastError.c_str(); }

int duck_batch_create_ex(const char *model_path, int num_envs, double dt, int iterations, int device, int fp64,
                         int specialized, int shared_memory, const duck_batch_options *options, duck_stream stream,
                         duck_batch **out) {
  return guarded([&] {
    require(out != nullptr && model_path != nullptr, "Invalid arguments");
    *out = nullptr;
    require(specialized || !shared_memory, "Shared memory requires the compact MicroDuck backend");
    require(num_envs > 0 && num_envs <= 65536 && dt > 0 && std::isfinite(dt) && iterations > 0,
            "Invalid batch parameters");
    const int maxPairs = options ? options->max_pairs : kReferencePairs;
    require(maxPairs >= 0 && maxPairs <= kMaxPairs, "max_pairs must be in [0, 128]");
    DeviceGuard guard(device);
    ParsedModel parsed = parseDuck(model_path, maxPairs);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    *out = fp64 ? create<double>(parsed, num_envs, dt, iterations, device, specialized, maxPairs, s)
                : create<float>(parsed, num_envs, dt, iterations, device, specialized, maxPairs, s);
  });
}

int duck_batch_create(const char *model_path, int num_envs, double dt, int iterations, int device, int fp64,
                      int specialized, int shared_memory, duck_stream stream, duck_batch **out) {
  return duck_batch_create_ex(model_path, num_envs, dt, iterations, device, fp64, specialized, shared_memory, nullptr,
                              stream, out);
}

void duck_batch_destroy(duck_batch *b) {
  if (!b) return;
  cudaSetDevice(b->device);
  if (b->ready) {
    cudaEventSynchronize(b->ready);
    cudaEventDestroy(b->ready);
  }
  cudaFree(b->devModel);
  cudaFree(b->points);
  cudaFree(b->records);
  cudaFree(b->envMass);
  cudaFree(b->envInertia);
  cudaFree(b->envFriction);
  delete b;
}

int duck_batch_info(const duck_batch *b, int32_t *out) {
  return guarded([&] {
    require(b && out, "Invalid arguments");
    int32_t v[10] = {b->n, b->nb, b->nj, b->bound, b->recordLength, b->fp64, b->device, b->teamsPerBlock, b->T,
                     b->smemPerBlock};
    std::memcpy(out, v, sizeof(v));
  });
}

int duck_batch_model_counts(const duck_batch *b, int32_t *out) {
  return guarded([&] {
    require(b && out, "Invalid arguments");
    const int ns = b->fp64 ? host<double>(b).dev.ns : host<float>(b).dev.ns;
    const int np = b->fp64 ? host<double>(b).dev.np : host<float>(b).dev.np;
    const int32_t v[4] = {b->nb, b->nj, ns, np};
    std::memcpy(out, v, sizeof(v));
  });
}

const char *duck_batch_joint_name(const duck_batch *b, int index) {
  if (!b || index < 0 || index >= int(b->names.size())) return nullptr;
  return b->names[index].c_str();
}

int duck_batch_reset(duck_batch *b, const uint8_t *mask, const void *q, const void *roots, duck_stream stream) {
  return guarded([&] {
    require(b && mask && roots && (q || b->nj == 0), "Invalid arguments");
    DeviceGuard guard(b->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    begin(b, s);
    if (b->fp64) launchReset<double>(b, mask, q, roots, 1, s);
    else launchReset<float>(b, mask, q, roots, 1, s);
    finish(b, s);
  });
}

int duck_batch_step(duck_batch *b, const void *target, const void *forces, int substeps, double kp, double limit,
                    duck_stream stream) {
  return guarded([&] {
    require(b && forces && (target || b->nj == 0), "Invalid arguments");
    // Zero selects the uncapped PD spring (extension.cu:290-294).
    require(substeps > 0 && kp >= 0 && std::isfinite(kp) && limit >= 0 && std::isfinite(limit), "Invalid controls");
    DeviceGuard guard(b->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    StepArgs args{target, forces, nullptr, substeps, kp, limit};
    begin(b, s);
    if (b->fp64) launchAdvance<double>(b, args, s);
    else launchAdvance<float>(b, args, s);
    finish(b, s);
  });
}

int duck_batch_step_motor(duck_batch *b, const void *motor, const void *forces, duck_stream stream) {
  return guarded([&] {
    require(b && forces && (motor || b->nj == 0), "Invalid arguments");
    DeviceGuard guard(b->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    StepArgs args{nullptr, forces, motor, 1, 0.0, 0.0};
    begin(b, s);
    if (b->fp64) launchAdvance<double>(b, args, s);
    else launchAdvance<float>(b, args, s);
    finish(b, s);
  });
}


int duck_batch_state(duck_batch *b, void *bodies, void *joints, void *diag, duck_stream stream) {
  return guarded([&] {
    require(b && bodies && diag && (joints || b->nj == 0), "Invalid arguments");
    DeviceGuard guard(b->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    begin(b, s);
    if (b->fp64) snapshot<double>(b, bodies, joints, diag, s);
    else snapshot<float>(b, bodies, joints, diag, s);
    finish(b, s);
  });
}

int duck_batch_contact_forces(duck_batch *b, void *out, int ground_only, duck_stream stream) {
  return guarded([&] {
    require(b && out, "Invalid arguments");
    DeviceGuard guard(b->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    begin(b, s);
    if (b->fp64) forcesLaunch<double>(b, out, ground_only, s);
    else forcesLaunch<float>(b, out, ground_only, s);
    finish(b, s);
  });
}

int duck_batch_self_contact_stats(duck_batch *b, void *out, duck_stream stream) {
  return guarded([&] {
    require(b && out, "Invalid arguments");
    DeviceGuard guard(b->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    begin(b, s);
    if (b->fp64) statsLaunch<double>(b, nullptr, out, s);
    else statsLaunch<float>(b, nullptr, out, s);
    finish(b, s);
  });
}

int duck_batch_contact_counts(duck_batch *b, void *out, duck_stream stream) {
  return guarded([&] {
    require(b && out, "Invalid arguments");
    DeviceGuard guard(b->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    begin(b, s);
    if (b->fp64) statsLaunch<double>(b, out, nullptr, s);
    else statsLaunch<float>(b, out, nullptr, s);
    finish(b, s);
  });
}

int duck_batch_generalized_loads(duck_batch *b, const void *offset, void *out, duck_stream stream) {
  return guarded([&] {
    require(b && offset && (out || b->nj == 0), "Invalid arguments");
    DeviceGuard guard(b->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    begin(b, s);
    if (b->fp64) loadsLaunch<double>(b, offset, out, s);
    else loadsLaunch<float>(b, offset, out, s);
    finish(b, s);
  });
}

int duck_batch_export(duck_batch *b, int first, int count, void *records, duck_stream stream) {
  return guarded([&] {
    require(b && records && first >= 0 && count >= 0 && first + count <= b->n, "Invalid environment range");
    DeviceGuard guard(b->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const size_t real = b->fp64 ? 8 : 4;
    begin(b, s);
    if (count > 0)
      check(cudaMemcpy2DAsync(records, b->recordLength * real,
                              static_cast<char *>(b->records) + size_t(first) * b->recordStride * real,
                              b->recordStride * real, b->recordLength * real, count, cudaMemcpyDeviceToDevice, s),
            "export copy");
    finish(b, s);
  });
}

int duck_batch_import(duck_batch *b, int first, int count, const void *records, duck_stream stream) {
  return guarded([&] {
    require(b && records && first >= 0 && count >= 0 && first + count <= b->n, "Invalid environment range");
    DeviceGuard guard(b->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const size_t real = b->fp64 ? 8 : 4;
    begin(b, s);
    if (count > 0)
      check(cudaMemcpy2DAsync(static_cast<char *>(b->records) + size_t(first) * b->recordStride * real,
                              b->recordStride * real, records, b->recordLength * real, b->recordLength * real, count,
                              cudaMemcpyDeviceToDevice, s),
            "import copy");
    finish(b, s);
  });
}

int duck_batch_contact_keys(duck_batch *b, int env, int32_t *keys, int capacity, int *count, duck_stream stream) {
  return guarded([&] {
    require(b && keys && count && env >= 0 && env < b->n && capacity >= 0, "Invalid arguments");
    DeviceGuard guard(b->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const size_t real = b->fp64 ? 8 : 4;
    std::vector<char> rec(b->recordLength * real);
    begin(b, s);
    check(cudaMemcpyAsync(rec.data(), static_cast<char *>(b->records) + size_t(env) * b->recordStride * real,
                          rec.size(), cudaMemcpyDeviceToHost, s),
          "contact copy");
    finish(b, s);
    check(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    auto value = [&](int i) {
      return b->fp64 ? reinterpret_cast<double *>(rec.data())[i] : double(reinterpret_cast<float *>(rec.data())[i]);
    };
    const int n = int(value(1));
    const int base = kRecHeader + kRecBody * b->nb + kRecJoint * b->nj;
    for (int i = 0; i < std::min(n, capacity); ++i)
      for (int k = 0; k < 5; ++k) keys[5 * i + k] = int32_t(value(base + kRecContact * i + (k == 4 ? 4 : k)));
    *count = n;
  });
}

int duck_batch_reference(duck_batch *b, const void *target, const void *forces, int substeps, double kp,
                         double limit, void *bodies, void *joints, void *diag) {
  return guarded([&] {
    require(b && forces && bodies && diag && (target || b->nj == 0) && (joints || b->nj == 0) && substeps > 0, "Invalid CPU reference inputs");
    DeviceGuard guard(b->device);
    const size_t real = b->fp64 ? 8 : 4;
    // A private one-environment batch sharing this batch's device model.
    duck_batch one = *b;
    one.n = 1;
    one.ready = nullptr;
    void *scratch = nullptr;
    const size_t bytes = size_t(one.recordStride) * real;
    size_t ioBytes = (b->nj + 3 + 13 * b->nb + 2 * b->nj + 6) * real;
    check(cudaMalloc(&scratch, bytes + ioBytes), "cudaMalloc reference");
    std::unique_ptr<void, void (*)(void *)> hold(scratch, [](void *p) { cudaFree(p); });
    one.records = scratch;
    char *io = static_cast<char *>(scratch) + bytes;
    char *dTarget = io, *dForces = io + b->nj * real, *dBodies = dForces + 3 * real,
         *dJoints = dBodies + 13 * b->nb * real, *dDiag = dJoints + 2 * b->nj * real;
    cudaStream_t s = nullptr;
    check(cudaMemcpy(dTarget, target, b->nj * real, cudaMemcpyHostToDevice), "copy target");
    check(cudaMemcpy(dForces, forces, 3 * real, cudaMemcpyHostToDevice), "copy forces");
    if (b->fp64) launchReset<double>(&one, nullptr, nullptr, nullptr, 0, s);
    else launchReset<float>(&one, nullptr, nullptr, nullptr, 0, s);
    StepArgs args{dTarget, dForces, nullptr, substeps, kp, limit};
    if (b->fp64) { launchAdvance<double>(&one, args, s); snapshot<double>(&one, dBodies, dJoints, dDiag, s); }
    else { launchAdvance<float>(&one, args, s); snapshot<float>(&one, dBodies, dJoints, dDiag, s); }
    check(cudaGetLastError(), "reference launch");
    check(cudaMemcpy(bodies, dBodies, 13 * b->nb * real, cudaMemcpyDeviceToHost), "copy bodies");
    check(cudaMemcpy(joints, dJoints, 2 * b->nj * real, cudaMemcpyDeviceToHost), "copy joints");
    check(cudaMemcpy(diag, dDiag, 6 * real, cudaMemcpyDeviceToHost), "copy diag");
    b->launches += one.launches - b->launches;
  });
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant of duck_batch_reference.
//
// duck_batch_reference takes its one-environment scratch record and staging
// buffers from cudaMalloc.  Some callers cannot allocate device memory at the
// moment they want this check: a host framework whose caching allocator owns
// the device memory and forbids raw cudaMalloc next to it, a process running
// under a fixed device-memory budget, or a real-time control loop that must
// not take the implicit synchronisation of cudaMalloc/cudaFree.  This variant
// keeps the scratch in a file-scope device array instead.  Every GPU that
// loads the library holds the array (kStaticScratchBytes) until exit; all
// calls share it and it keeps the previous call's contents, so the record is
// cleared on every call, and calls that overlap on the GPU race.  The call is
// synchronous like duck_batch_reference: it copies from and to host memory
// with cudaMemcpy and works on the legacy default stream.
static constexpr size_t kStaticScratchBytes = 32 * 1024;
static __device__ __align__(256) unsigned char duckStaticScratch[kStaticScratchBytes];

namespace {
std::mutex staticScratchMutex;
void *staticScratchAddress[64] = {};

// Device address of duckStaticScratch on `device` (current), resolved once per
// device at its first call: host code cannot use the symbol itself, which
// names a host-side stand-in, not device memory.  The cached address belongs
// to the device's primary context: a cudaDeviceReset of that device (which
// also invalidates every batch on it) leaves it stale, so a process must not
// use this entry point on a device after resetting it.
void *staticScratch(int device) {
  require(device >= 0 && device < 64, "Device index out of range");
  std::lock_guard<std::mutex> lock(staticScratchMutex);
  if (!staticScratchAddress[device]) {
    void *ptr = nullptr;
    check(cudaGetSymbolAddress(&ptr, duckStaticScratch), "cudaGetSymbolAddress");
    staticScratchAddress[device] = ptr;
  }
  return staticScratchAddress[device];
}

template <class R>
void referenceStatic(duck_batch *b, char *scratch, size_t recordBytes, const StepArgs &stepArgs, char *dBodies,
                     char *dJoints, char *dDiag) {
  const DevModel<R> *m = static_cast<const DevModel<R> *>(b->devModel);
  const R *pts = static_cast<const R *>(b->points);
  R *rec = reinterpret_cast<R *>(scratch);
  const int stride = b->recordStride;
  // The one-environment record is environment 0 of the parameter arrays, as
  // in duck_batch_reference's private batch.
  StepArgs args = stepArgs;
  args.mass = b->envMass;
  args.inertia = b->envInertia;
  args.friction = b->envFriction;
  check(cudaMemset(scratch, 0, recordBytes), "cudaMemset scratch record");
  resetKernel<R><<<1, 128>>>(m, rec, stride, 1, nullptr, nullptr, nullptr, 0);
  withAdvance<R>(b, [&](auto kernel) { kernel<<<1, 32, b->smemPerBlock>>>(m, pts, rec, stride, 1, b->layout, args); });
  snapshotKernel<R><<<blocksFor(b->nb + b->nj + 1, 256), 256>>>(m, rec, stride, 1, reinterpret_cast<R *>(dBodies), reinterpret_cast<R *>(dJoints),
                               reinterpret_cast<R *>(dDiag));
  check(cudaGetLastError(), "static reference launch");
  b->launches += 3;
}
}  // namespace

extern "C" {

int duck_batch_reference_static(duck_batch *b, const void *target, const void *forces, int substeps, double kp,
                                 double limit, void *bodies, void *joints, void *diag) {
  return guarded([&] {
    require(b && forces && bodies && diag && (target || b->nj == 0) && (joints || b->nj == 0) && substeps > 0,
            "Invalid CPU reference inputs");
    require(kp >= 0 && std::isfinite(kp) && limit >= 0 && std::isfinite(limit), "Invalid controls");
    DeviceGuard guard(b->device);
    const size_t real = b->fp64 ? 8 : 4;
    const size_t recordBytes = size_t(b->recordStride) * real;
    const size_t ioBytes = size_t(b->nj + 3 + 13 * b->nb + 2 * b->nj + 6) * real;
    if (recordBytes + ioBytes > kStaticScratchBytes)
      throw std::invalid_argument("Model too large for the static reference scratch: needs " +
                                  std::to_string(recordBytes + ioBytes) + " bytes, the library reserves " +
                                  std::to_string(kStaticScratchBytes));
    char *scratch = static_cast<char *>(staticScratch(b->device));
    char *io = scratch + recordBytes;
    char *dTarget = io, *dForces = io + b->nj * real, *dBodies = dForces + 3 * real,
         *dJoints = dBodies + 13 * b->nb * real, *dDiag = dJoints + 2 * b->nj * real;
    if (b->nj) check(cudaMemcpy(dTarget, target, b->nj * real, cudaMemcpyHostToDevice), "copy target");
    check(cudaMemcpy(dForces, forces, 3 * real, cudaMemcpyHostToDevice), "copy forces");
    StepArgs args{dTarget, dForces, nullptr, substeps, kp, limit};
    if (b->fp64) referenceStatic<double>(b, scratch, recordBytes, args, dBodies, dJoints, dDiag);
    else referenceStatic<float>(b, scratch, recordBytes, args, dBodies, dJoints, dDiag);
    check(cudaMemcpy(bodies, dBodies, 13 * b->nb * real, cudaMemcpyDeviceToHost), "copy bodies");
    if (b->nj) check(cudaMemcpy(joints, dJoints, 2 * b->nj * real, cudaMemcpyDeviceToHost), "copy joints");
    check(cudaMemcpy(diag, dDiag, 6 * real, cudaMemcpyDeviceToHost), "copy diag");
  });
}

}  // extern "C"

namespace {
EnvKernelParams envParams(const duck_batch *b, const duck_env_params *p) {
  require(p != nullptr, "Invalid arguments");
  require(p->task == 0 || p->task == 1, "Unknown task");
  require(p->control_dt > 0 && p->tracking_sigma > 0 && p->gait_period > 0 && p->max_episode_length > 0,
          "Invalid environment parameters");
  EnvKernelParams k{};
  k.task = p->task;
  k.filter = p->filter ? 1 : 0;
  k.maxEpisode = p->max_episode_length;
  k.nj = b->nj;
  k.obsDim = 10 + 3 * b->nj + (p->task == 1 ? 6 : 0) + (k.filter ? 2 : 0);
  k.rootHeight = p->root_height;
  k.tilt = float(p->tilt);
  k.controlDt = p->control_dt;
  k.velocityAlpha = p->velocity_alpha;
  k.trackingWeight = p->tracking_weight;
  k.headingWeight = p->heading_weight;
  k.sigma2 = p->tracking_sigma * p->tracking_sigma;
  k.phaseRate = 2 * 3.14159265358979323846 / p->gait_period;
  for (int i = 0; i < 4; ++i) k.iquat[i] = p->iquat[i];
  k.gait = p->gait;
  k.footClearance = p->foot_clearance;
  k.loadTransfer = p->load_transfer;
  if (p->gait) require(p->gait_table != nullptr && p->gait_samples > 0, "Gait shaping needs the gait table");
  if (p->foot_clearance) require(p->foot_xyz != nullptr && p->foot_points > 0, "Foot clearance needs foot points");
  if (p->foot_clearance || p->load_transfer)
    require(p->foot_body[0] > 0 && p->foot_body[0] < b->nb && p->foot_body[1] > 0 && p->foot_body[1] < b->nb &&
                (!p->load_transfer || p->mass > 0),
            "Invalid foot bodies or mass");
  k.gaitSamples = p->gait_samples;
  k.footPoints = p->foot_points;
  k.footBody[0] = p->foot_body[0];
  k.footBody[1] = p->foot_body[1];
  k.gaitPeriod = p->gait_period;
  k.gaitLift = p->gait_lift;
  k.massG = p->mass * 9.81;
  k.gaitTable = p->gait_table;
  k.footXyz = p->foot_xyz;
  return k;
}
}  // namespace

extern "C" {

int duck_env_obs_dim(const duck_batch *b, const duck_env_params *p) {
  if (!b || !p) return -1;
  return 10 + 3 * b->nj + (p->task == 1 ? 6 : 0) + (p->filter ? 2 : 0);
}

int duck_env_targets(duck_batch *b, const void *actions, double scale, const void *home, const void *lower,
                     const void *upper, void *a_out, void *target_out, duck_stream stream) {
  return guarded([&] {
    require(b && actions && home && lower && upper && a_out && target_out, "Invalid arguments");
    DeviceGuard guard(b->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int items = b->n * b->nj;
    if (items == 0) return;
    if (b->fp64)
      envTargetsKernel<double><<<blocksFor(items, 256), 256, 0, s>>>(
          b->n, b->nj, static_cast<const double *>(actions), scale, static_cast<const double *>(home), static_cast<const double *>(lower),
          static_cast<const double *>(upper), static_cast<double *>(a_out), static_cast<double *>(target_out));
    else
      envTargetsKernel<float><<<blocksFor(items, 256), 256, 0, s>>>(
          b->n, b->nj, static_cast<const float *>(actions), float(scale), static_cast<const float *>(home), static_cast<const float *>(lower),
          static_cast<const float *>(upper), static_cast<float *>(a_out), static_cast<float *>(target_out));
    ++b->launches;
    check(cudaGetLastError(), "env targets");
  });
}

int duck_env_reference_targets(duck_batch *b, const duck_env_params *params, const void *actions, double scale,
                               const void *home, const void *lower, const void *upper, const int64_t *episode_length,
                               const void *commands, void *a_out, void *target_out, duck_stream stream) {
  return guarded([&] {
    require(b && actions && home && lower && upper && episode_length && commands && a_out && target_out,
            "Invalid arguments");
    const EnvKernelParams k = envParams(b, params);
    DeviceGuard guard(b->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int items = b->n * b->nj;
    if (items == 0) return;
    auto run = [&](auto zero) {
      using R = decltype(zero);
      envGaitTargetsKernel<R><<<blocksFor(items, 256), 256, 0, s>>>(
          b->n, k, static_cast<const R *>(actions), R(scale), static_cast<const R *>(home),
          static_cast<const R *>(lower), static_cast<const R *>(upper),
          reinterpret_cast<const long long *>(episode_length), static_cast<const R *>(commands),
          static_cast<R *>(a_out), static_cast<R *>(target_out));
    };
    if (b->fp64) run(0.0); else run(0.0f);
    ++b->launches;
    check(cudaGetLastError(), "env reference targets");
  });
}

int duck_env_post_step(duck_batch *b, const duck_env_params *params, const void *home, const void *a,
                       void *prev_actions, int64_t *episode_length, float *returns, const void *commands,
                       void *filtered, float *obs, float *reward, uint8_t *failed, uint8_t *timeout,
                       uint8_t *done, void *diag, float *tracking, duck_stream stream) {
  return guarded([&] {
    require(b && home && a && prev_actions && episode_length && returns && commands && filtered && obs && reward &&
                failed && timeout && done,
            "Invalid arguments");
    const EnvKernelParams k = envParams(b, params);
    DeviceGuard guard(b->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    begin(b, s);
    auto run = [&](auto zero) {
      using R = decltype(zero);
      envPostStepKernel<R><<<blocksFor(b->n, 128), 128, 0, s>>>(
          static_cast<const DevModel<R> *>(b->devModel), static_cast<const R *>(b->records), b->recordStride, b->n,
          k, static_cast<const R *>(home), static_cast<const R *>(a), static_cast<R *>(prev_actions),
          reinterpret_cast<long long *>(episode_length), returns, static_cast<const R *>(commands),
          static_cast<R *>(filtered), obs, reward, reinterpret_cast<bool *>(failed),
          reinterpret_cast<bool *>(timeout), reinterpret_cast<bool *>(done), static_cast<R *>(diag), tracking);
    };
    if (b->fp64) run(0.0); else run(0.0f);
    ++b->launches;
    finish(b, s);
  });
}

int duck_env_observe(duck_batch *b, const duck_env_params *params, const void *home, const void *actions,
                     const int64_t *episode_length, const void *commands, const void *filtered, float *obs,
                     duck_stream stream) {
  return guarded([&] {
    require(b && home && actions && episode_length && commands && filtered && obs, "Invalid arguments");
    const EnvKernelParams k = envParams(b, params);
    DeviceGuard guard(b->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    begin(b, s);
    auto run = [&](auto zero) {
      using R = decltype(zero);
      envObserveKernel<R><<<blocksFor(b->n, 128), 128, 0, s>>>(
          static_cast<const DevModel<R> *>(b->devModel), static_cast<const R *>(b->records), b->recordStride, b->n,
          k, static_cast<const R *>(home), static_cast<const R *>(actions),
          reinterpret_cast<const long long *>(episode_length), static_cast<const R *>(commands),
          static_cast<const R *>(filtered), obs);
    };
    if (b->fp64) run(0.0); else run(0.0f);
    ++b->launches;
    finish(b, s);
  });
}

int duck_env_reset_buffers(duck_batch *b, const uint8_t *mask, void *prev_actions, void *forces,
                           int64_t *episode_length, float *returns, void *filtered, void *commands,
                           const void *new_commands, duck_stream stream) {
  return guarded([&] {
    require(b && mask && prev_actions && forces && episode_length && returns && filtered && commands,
            "Invalid arguments");
    DeviceGuard guard(b->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    auto run = [&](auto zero) {
      using R = decltype(zero);
      envResetBuffersKernel<R><<<blocksFor(b->n, 128), 128, 0, s>>>(
          b->n, b->nj, reinterpret_cast<const bool *>(mask), static_cast<R *>(prev_actions), static_cast<R *>(forces),
          reinterpret_cast<long long *>(episode_length), returns, static_cast<R *>(filtered),
          static_cast<R *>(commands), static_cast<const R *>(new_commands));
    };
    if (b->fp64) run(0.0); else run(0.0f);
    ++b->launches;
    check(cudaGetLastError(), "env reset buffers");
  });
}

}  // extern "C"

namespace {
BamKernelParams bamParams(const duck_batch *b, const duck_bam_params *p) {
  require(p != nullptr, "Invalid arguments");
  require(b->nj > 0 && b->nj <= 32, "The BAM environment needs 1..32 joints");
  require(p->lag >= 0 && p->decimation >= 1 && p->max_episode_length > 0 && p->dt > 0 && p->step_dt > 0,
          "Invalid BAM control settings");
  require(p->foot_body[0] > 0 && p->foot_body[0] < b->nb && p->foot_body[1] > 0 && p->foot_body[1] < b->nb,
          "Foot body index out of range");
  require(p->vin_min > 0 && p->R > 0 && p->dtheta_stribeck > 0 && p->force_limit >= 0, "Invalid servo parameters");
  int heads = 0;
  for (int j = 0; j < b->nj; ++j) heads += (p->head_mask >> j) & 1;
  require(heads == 4, "The walking reward needs exactly four head joints");
  BamKernelParams k{};
  k.nj = b->nj;
  k.lag = p->lag;
  k.maxEpisode = p->max_episode_length;
  k.sourceIteration = p->source_iteration;
  k.neutralHead = p->neutral_head;
  k.headingHold = p->heading_hold;
  k.reward = p->reward_enabled;
  k.headMask = int(p->head_mask);
  k.extras = (p->head_stability ? xHeadStability : 0) | (p->mean_velocity ? xMeanVelocity : 0) |
             (p->heading_reward ? xHeading : 0);
  k.overrideMask = int(p->override_mask);
  k.criticDim = 34 + 3 * b->nj + (p->mean_velocity ? 3 : 0) + (p->heading_reward ? 1 : 0);
  k.footBody[0] = p->foot_body[0];
  k.footBody[1] = p->foot_body[1];
  k.dt = p->dt; k.stepDt = p->step_dt; k.kpFw = p->kp_fw; k.vin = p->vin; k.vinDrop = p->vin_drop_gain;
  k.vinMin = p->vin_min; k.forceLimit = p->force_limit;
  k.kt = p->kt; k.res = p->R; k.fBase = p->friction_base; k.fStribeck = p->friction_stribeck;
  k.lfe = p->load_friction_external; k.lfm = p->load_friction_motor; k.lfes = p->load_friction_external_stribeck;
  k.lfms = p->load_friction_motor_stribeck; k.lfeq = p->load_friction_external_quad;
  k.lfmq = p->load_friction_motor_quad; k.dthetaStribeck = p->dtheta_stribeck; k.alpha = p->alpha;
  k.fViscous = p->friction_viscous;
  for (int i = 0; i < 4; ++i) k.iquat[i] = p->root_iquat[i];
  for (int f = 0; f < 2; ++f)
    for (int i = 0; i < 3; ++i) k.site[f][i] = p->foot_site[f][i];
  k.linVar = p->linear_variance; k.vertVar = p->vertical_variance; k.meanAlpha = p->mean_velocity_alpha;
  k.meanVar = p->mean_velocity_variance; k.meanWeight = p->mean_velocity_weight;
  k.headingWeight = p->heading_reward_weight; k.headingVar = p->heading_reward_variance;
  k.headPosWeight = p->head_position_weight; k.headVelWeight = p->head_velocity_weight;
  k.tiltLimit = p->tilt_limit;
  for (int t = 0; t < 15; ++t) k.overrides[t] = p->overrides[t];
  for (int j = 0; j < 32; ++j) {
    k.stand[j] = p->stand_std[j];
    k.walk[j] = p->walk_std[j];
    k.soft[j][0] = p->soft_limits[j][0];
    k.soft[j][1] = p->soft_limits[j][1];
  }
  return k;
}

template <class R> BamBuffers<R> bamBuffers(const duck_bam_buffers *x) {
  require(x != nullptr, "Invalid arguments");
  const void *need[] = {x->home, x->root_offset, x->zero_forces, x->action, x->old_action, x->previous_motor,
                        x->previous_applied, x->observed_velocity, x->command, x->mean_velocity_world,
                        x->target_yaw, x->self_contacts, x->self_penetration, x->air_time, x->contact_time,
                        x->peak_height, x->contact_force, x->joints, x->head_ema, x->target_history, x->motor,
                        x->features, x->terms, x->contact, x->history_initialized, x->done, x->timeout,
                        x->failed, x->episode_length, x->counters, x->obs_actor, x->obs_critic, x->reward,
                        x->servo_supply};
  for (const void *ptr : need) require(ptr != nullptr, "Missing BAM buffer");
  BamBuffers<R> B;
  B.home = static_cast<const R *>(x->home);
  B.rootOffset = static_cast<const R *>(x->root_offset);
  B.action = static_cast<R *>(x->action);
  B.oldAction = static_cast<R *>(x->old_action);
  B.prevMotor = static_cast<R *>(x->previous_motor);
  B.prevApplied = static_cast<R *>(x->previous_applied);
  B.observedVelocity = static_cast<R *>(x->observed_velocity);
  B.command = static_cast<R *>(x->command);
  B.meanVelocity = static_cast<R *>(x->mean_velocity_world);
  B.targetYaw = static_cast<R *>(x->target_yaw);
  B.airTime = static_cast<R *>(x->air_time);
  B.contactTime = static_cast<R *>(x->contact_time);
  B.contactForce = static_cast<R *>(x->contact_force);
  B.selfContacts = static_cast<R *>(x->self_contacts);
  B.selfPenetration = static_cast<R *>(x->self_penetration);
  B.joints = static_cast<R *>(x->joints);
  B.headEma = static_cast<R *>(x->head_ema);
  B.peakHeight = static_cast<R *>(x->peak_height);
  B.history = static_cast<R *>(x->target_history);
  B.motor = static_cast<R *>(x->motor);
  B.features = static_cast<R *>(x->features);
  B.terms = static_cast<R *>(x->terms);
  B.servoSupply = static_cast<R *>(x->servo_supply);
  B.contact = reinterpret_cast<bool *>(x->contact);
  B.histInit = reinterpret_cast<bool *>(x->history_initialized);
  B.done = reinterpret_cast<bool *>(x->done);
  B.timeout = reinterpret_cast<bool *>(x->timeout);
  B.failed = reinterpret_cast<bool *>(x->failed);
  B.episodeLength = reinterpret_cast<long long *>(x->episode_length);
  B.counters = x->counters;
  B.obsActor = x->obs_actor;
  B.obsCritic = x->obs_critic;
  B.reward = x->reward;
  return B;
}

enum BamPart { kBamBegin = 1, kBamSubstep = 2, kBamFinish = 4, kBamServoOnly = 8 };

template <class R>
void bamRun(duck_batch *b, const BamKernelParams &k, const duck_bam_buffers *x, const void *actions, int parts,
            int substeps, cudaStream_t s) {
  static_assert(kMaxBodies * 18 * 32 * sizeof(double) <= 160 * 1024, "RNEA shared arrays");
  // Raise the loads kernel's shared-memory limit when a model needs more than
  // any before (the first, eager step does it, so captures never need to).
  static int rneaLimit[2][64] = {};
  const int need = int(18 * b->nb * 32 * sizeof(R));
  int &limit = rneaLimit[sizeof(R) == 8][b->device & 63];
  if (need > limit) {
    check(cudaFuncSetAttribute(bamLoadsKernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, need),
          "cudaFuncSetAttribute");
    limit = need;
  }
  BamBuffers<R> B = bamBuffers<R>(x);
  B.envMass = static_cast<const R *>(b->envMass);
  B.envInertia = static_cast<const R *>(b->envInertia);
  const DevModel<R> *m = static_cast<const DevModel<R> *>(b->devModel);
  const R *rec = static_cast<const R *>(b->records);
  const int grid = blocksFor(b->n, 128);
  if (parts & kBamBegin) {
    bamBeginKernel<R><<<grid, 128, 0, s>>>(k, B, b->n, static_cast<const R *>(actions));
    ++b->launches;
  }
  const size_t rneaBytes = size_t(18) * b->nb * 32 * sizeof(R);
  auto servo = [&] {
    bamLoadsKernel<R><<<blocksFor(b->n, 32), 32, rneaBytes, s>>>(m, rec, b->recordStride, b->n, k, B);
    bamServoJointKernel<R><<<blocksFor(size_t(b->n) * b->nj, 128), 128, 0, s>>>(m, rec, b->recordStride, b->n, k, B);
    b->launches += 2;
  };
  if (parts & kBamServoOnly) servo();
  if (parts & kBamSubstep) {
    for (int i = 0; i < substeps; ++i) {
      servo();
      StepArgs args{nullptr, x->zero_forces, x->motor, 1, 0.0, 0.0};
      launchAdvance<R>(b, args, s);
      bamAfterKernel<R><<<grid, 128, 0, s>>>(m, rec, b->recordStride, b->n, k, B);
      ++b->launches;
    }
  }
  if (parts & kBamFinish) {
    bamControlKernel<R><<<grid, 128, 0, s>>>(m, rec, b->recordStride, b->n, k, B, 0, nullptr);
    ++b->launches;
  }
}

int bamCall(duck_batch *b, const duck_bam_params *params, const duck_bam_buffers *x, const void *actions,
            int parts, duck_stream stream) {
  return guarded([&] {
    require(b && x, "Invalid arguments");
    require(!(parts & kBamBegin) || actions, "Missing actions");
    const BamKernelParams k = bamParams(b, params);
    DeviceGuard guard(b->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    begin(b, s);
    if (b->fp64) bamRun<double>(b, k, x, actions, parts, params->decimation, s);
    else bamRun<float>(b, k, x, actions, parts, params->decimation, s);
    finish(b, s);
  });
}
}  // namespace

extern "C" {

int duck_bam_critic_dim(const duck_batch *b, const duck_bam_params *p) {
  if (!b || !p) return -1;
  return 34 + 3 * b->nj + (p->mean_velocity ? 3 : 0) + (p->heading_reward ? 1 : 0);
}

int duck_bam_step(duck_batch *b, const duck_bam_params *p, const duck_bam_buffers *x, const void *actions,
                  duck_stream stream) {
  return bamCall(b, p, x, actions, kBamBegin | kBamSubstep | kBamFinish, stream);
}

int duck_bam_begin(duck_batch *b, const duck_bam_params *p, const duck_bam_buffers *x, const void *actions,
                   duck_stream stream) {
  return bamCall(b, p, x, actions, kBamBegin, stream);
}

int duck_bam_substep(duck_batch *b, const duck_bam_params *p, const duck_bam_buffers *x, duck_stream stream) {
  if (!p) return bamCall(b, p, x, nullptr, 0, stream);
  duck_bam_params one = *p;
  one.decimation = 1;
  return bamCall(b, &one, x, nullptr, kBamSubstep, stream);
}

int duck_bam_finish(duck_batch *b, const duck_bam_params *p, const duck_bam_buffers *x, duck_stream stream) {
  return bamCall(b, p, x, nullptr, kBamFinish, stream);
}

int duck_bam_servo(duck_batch *b, const duck_bam_params *p, const duck_bam_buffers *x, duck_stream stream) {
  return bamCall(b, p, x, nullptr, kBamServoOnly, stream);
}

int duck_bam_reset_buffers(duck_batch *b, const duck_bam_params *p, const duck_bam_buffers *x, const uint8_t *mask,
                           duck_stream stream) {
  return guarded([&] {
    require(b && x && mask, "Invalid arguments");
    const BamKernelParams k = bamParams(b, p);
    DeviceGuard guard(b->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    auto run = [&](auto zero) {
      using R = decltype(zero);
      bamResetKernel<R><<<blocksFor(b->n, 128), 128, 0, s>>>(k, bamBuffers<R>(x), b->n,
                                                              reinterpret_cast<const bool *>(mask));
    };
    if (b->fp64) run(0.0); else run(0.0f);
    ++b->launches;
    check(cudaGetLastError(), "bam reset buffers");
  });
}

int duck_bam_observe(duck_batch *b, const duck_bam_params *p, const duck_bam_buffers *x, const uint8_t *mask,
                     int update_heading, duck_stream stream) {
  return guarded([&] {
    require(b && x, "Invalid arguments");
    const BamKernelParams k = bamParams(b, p);
    DeviceGuard guard(b->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    begin(b, s);
    auto run = [&](auto zero) {
      using R = decltype(zero);
      bamControlKernel<R><<<blocksFor(b->n, 128), 128, 0, s>>>(
          static_cast<const DevModel<R> *>(b->devModel), static_cast<const R *>(b->records), b->recordStride, b->n,
          k, bamBuffers<R>(x), update_heading ? 1 : 2, reinterpret_cast<const bool *>(mask));
    };
    if (b->fp64) run(0.0); else run(0.0f);
    ++b->launches;
    finish(b, s);
  });
}

int duck_batch_set_parameters(duck_batch *b, const void *mass, const void *inertia, const void *friction,
                              duck_stream stream) {
  return guarded([&] {
    require(b != nullptr, "Invalid arguments");
    DeviceGuard guard(b->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const size_t real = b->fp64 ? 8 : 4;
    const int ns = b->fp64 ? host<double>(b).dev.ns : host<float>(b).dev.ns;
    begin(b, s);
    auto install = [&](void *&slot, const void *src, size_t count, const char *what) {
      if (!src) {
        if (slot) {
          check(cudaStreamSynchronize(s), "cudaStreamSynchronize");
          check(cudaFree(slot), "cudaFree");
          slot = nullptr;
        }
        return;
      }
      if (!slot) check(cudaMalloc(&slot, count * real), what);
      check(cudaMemcpyAsync(slot, src, count * real, cudaMemcpyDeviceToDevice, s), what);
    };
    install(b->envMass, mass, size_t(b->n) * b->nb, "per-env masses");
    install(b->envInertia, inertia, size_t(b->n) * b->nb * 3, "per-env inertias");
    install(b->envFriction, friction, size_t(b->n) * ns, "per-env frictions");
    auto run = [&](auto zero) {
      using R = decltype(zero);
      checkParametersKernel<R><<<blocksFor(b->n, 128), 128, 0, s>>>(
          static_cast<const DevModel<R> *>(b->devModel), static_cast<R *>(b->records), b->recordStride, b->n,
          static_cast<const R *>(b->envMass), static_cast<const R *>(b->envInertia),
          static_cast<const R *>(b->envFriction));
    };
    if (b->fp64) run(0.0); else run(0.0f);
    ++b->launches;
    finish(b, s);
  });
}

int64_t duck_batch_launches(const duck_batch *b) { return b ? b->launches : 0; }

int duck_ppo_loss_scratch(int batch, int actions) {
  if (batch <= 0 || actions <= 0 || actions > kPpoMaxActions) return -1;
  return ((batch + kPpoThreads - 1) / kPpoThreads) * ppoPartials(actions);
}

int duck_ppo_loss(int batch, int actions, const float *mu, const float *std, const float *value, const float *act,
                  const float *old_log_prob, const float *old_mu, const float *old_sigma, const float *target_value,
                  const float *returns, const float *advantage, double clip, double value_coef,
                  double entropy_coef, float *scratch, float *out, float *grad_mu, float *grad_std,
                  float *grad_value, duck_stream stream) {
  return guarded([&] {
    require(batch > 0 && actions > 0 && actions <= kPpoMaxActions, "Invalid PPO batch or action count");
    require(mu && std && value && act && old_log_prob && old_mu && old_sigma && target_value && returns && advantage &&
                scratch && out && grad_mu && grad_std && grad_value,
            "Invalid arguments");
    require(clip >= 0 && std::isfinite(clip) && std::isfinite(value_coef) && std::isfinite(entropy_coef),
            "Invalid PPO coefficients");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    PpoLossArgs a{batch, actions, mu, std, value, act, old_log_prob, old_mu, old_sigma, target_value, returns,
                  advantage, float(clip), float(value_coef), float(entropy_coef), scratch, out, grad_mu,
                  grad_std, grad_value};
    const int blocks = (batch + kPpoThreads - 1) / kPpoThreads;
    if (actions <= 16) {
      ppoLossRows<16><<<blocks, kPpoThreads, 0, s>>>(a);
      ppoLossFinish<16><<<1, kPpoThreads, 0, s>>>(a, blocks);
    } else {
      ppoLossRows<32><<<blocks, kPpoThreads, 0, s>>>(a);
      ppoLossFinish<32><<<1, kPpoThreads, 0, s>>>(a, blocks);
    }
    check(cudaGetLastError(), "PPO loss launch");
  });
}

int duck_fp32_peak(int device, int iterations, double *tflops, duck_stream stream) {
  return guarded([&] {
    require(tflops && iterations > 0, "Invalid arguments");
    DeviceGuard guard(device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int sms = 0;
    check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device), "cudaDeviceGetAttribute");
    float *sink = nullptr;
    check(cudaMalloc(&sink, sizeof(float)), "cudaMalloc sink");
    std::unique_ptr<float, void (*)(float *)> hold(sink, [](float *p) { cudaFree(p); });
    cudaEvent_t start, stop;
    check(cudaEventCreate(&start), "cudaEventCreate");
    check(cudaEventCreate(&stop), "cudaEventCreate");
    const int blocks = sms * 8, threads = 256;
    fmaPeakKernel<<<blocks, threads, 0, s>>>(sink, iterations / 10 + 1, 1.0f);
    check(cudaEventRecord(start, s), "cudaEventRecord");
    fmaPeakKernel<<<blocks, threads, 0, s>>>(sink, iterations, 1.0f);
    check(cudaEventRecord(stop, s), "cudaEventRecord");
    check(cudaEventSynchronize(stop), "cudaEventSynchronize");
    float ms = 0;
    check(cudaEventElapsedTime(&ms, start, stop), "cudaEventElapsedTime");
    cudaEventDestroy(start);
    cudaEventDestroy(stop);
    *tflops = 2.0 * 8.0 * double(iterations) * blocks * threads / (ms * 1e-3) / 1e12;
  });
}

}  // extern "C"
