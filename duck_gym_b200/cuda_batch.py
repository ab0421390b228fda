"""Python binding of the C ABI with the reference's ``CudaBatch`` API.

Mirrors ``_duck_cuda.CudaBatch`` (src/cuda/extension.cu:436-452):

    CudaBatch(model, num_envs, dt=.001, iterations=200, device=0, fp64=False,
              specialized=False, shared_memory=False)
    .reset(mask[E] bool, q[E,J], root[E,6])
    .step(target[E,J], forces[E,3], substeps, kp, limit)
    .step_motor(motor[E,J,3], forces[E,3])
    .state() -> [bodies[E,B,13], joints[E,J,2], diag[E,6]]
    .contact_forces(ground_only=False) -> [E,B,3]
    .self_contact_stats() -> [E,2]
    .contact_counts() -> [E,2]
    .generalized_loads(offset[E,3]) -> [E,J,3]
    .reference(target[J] cpu, forces[3] cpu, substeps, kp, limit)
    .joint_names

Same conventions as the reference (extension.cu:203-213): inputs must be CUDA
tensors on the batch's device with the batch dtype, contiguous and of exact
shape, else ``RuntimeError``; each input is recorded on the current stream;
outputs are fresh tensors; work is ordered on the current torch stream and
serialised across streams by the library's private event.  There is no CPU
fallback: constructing a batch without the compiled library raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

from . import build as _build

_lib = None


def library():
    """Load ``libduck_b200.so`` (built in-tree by ``duck_gym_b200.build``)."""
    global _lib
    if _lib is None:
        path = _build.LIB_PATH
        if not path.exists():
            raise RuntimeError(
                f"{path} is missing: build it with `python -m duck_gym_b200.build` "
                "(the CUDA path has no fallback)")
        lib = ctypes.CDLL(str(path))
        P, I, D = ctypes.c_void_p, ctypes.c_int, ctypes.c_double
        lib.duck_last_error.restype = ctypes.c_char_p
        lib.duck_batch_create.argtypes = [ctypes.c_char_p, I, D, I, I, I, I, I, P, ctypes.POINTER(P)]
        lib.duck_batch_create_ex.argtypes = [ctypes.c_char_p, I, D, I, I, I, I, I, P, P, ctypes.POINTER(P)]
        lib.duck_batch_destroy.argtypes = [P]
        lib.duck_batch_destroy.restype = None
        lib.duck_batch_info.argtypes = [P, P]
        lib.duck_batch_joint_name.argtypes = [P, I]
        lib.duck_batch_joint_name.restype = ctypes.c_char_p
        lib.duck_batch_reset.argtypes = [P, P, P, P, P]
        lib.duck_batch_step.argtypes = [P, P, P, I, D, D, P]
        lib.duck_batch_step_motor.argtypes = [P, P, P, P]
        lib.duck_batch_state.argtypes = [P, P, P, P, P]
        lib.duck_batch_contact_forces.argtypes = [P, P, I, P]
        lib.duck_batch_self_contact_stats.argtypes = [P, P, P]
        lib.duck_batch_contact_counts.argtypes = [P, P, P]
        lib.duck_batch_generalized_loads.argtypes = [P, P, P, P]
        lib.duck_batch_reference.argtypes = [P, P, P, I, D, D, P, P, P]
        lib.duck_batch_export.argtypes = [P, I, I, P, P]
        lib.duck_batch_import.argtypes = [P, I, I, P, P]
        lib.duck_batch_contact_keys.argtypes = [P, I, P, I, ctypes.POINTER(I), P]
        lib.duck_batch_set_parameters.argtypes = [P, P, P, P, P]
        lib.duck_batch_model_counts.argtypes = [P, P]
        lib.duck_batch_launches.argtypes = [P]
        lib.duck_batch_launches.restype = ctypes.c_int64
        lib.duck_fp32_peak.argtypes = [I, I, ctypes.POINTER(D), P]
        lib.duck_ppo_loss_scratch.argtypes = [I, I]
        lib.duck_ppo_loss.argtypes = [I, I] + [P] * 10 + [D, D, D] + [P] * 5 + [P]
        lib.duck_env_obs_dim.argtypes = [P, P]
        lib.duck_env_targets.argtypes = [P, P, D, P, P, P, P, P, P]
        lib.duck_env_reference_targets.argtypes = [P, P, P, D, P, P, P, P, P, P, P, P]
        lib.duck_env_post_step.argtypes = [P] * 17
        lib.duck_env_observe.argtypes = [P] * 9
        lib.duck_env_reset_buffers.argtypes = [P] * 10
        lib.duck_bam_critic_dim.argtypes = [P, P]
        for name in ("duck_bam_step", "duck_bam_begin"):
            getattr(lib, name).argtypes = [P, P, P, P, P]
        for name in ("duck_bam_substep", "duck_bam_finish", "duck_bam_servo"):
            getattr(lib, name).argtypes = [P, P, P, P]
        lib.duck_bam_reset_buffers.argtypes = [P, P, P, P, P]
        lib.duck_bam_observe.argtypes = [P, P, P, P, I, P]
        for name in ("duck_batch_create", "duck_batch_create_ex", "duck_batch_set_parameters", "duck_batch_model_counts",
                     "duck_batch_info", "duck_batch_reset", "duck_batch_step",
                     "duck_batch_step_motor", "duck_batch_state", "duck_batch_contact_forces",
                     "duck_batch_self_contact_stats", "duck_batch_contact_counts",
                     "duck_batch_generalized_loads", "duck_batch_reference", "duck_batch_export",
                     "duck_batch_import", "duck_batch_contact_keys", "duck_fp32_peak", "duck_env_obs_dim",
                     "duck_env_targets", "duck_env_reference_targets", "duck_env_post_step", "duck_env_observe", "duck_env_reset_buffers",
                     "duck_bam_critic_dim", "duck_bam_step", "duck_bam_begin", "duck_bam_substep", "duck_bam_finish",
                     "duck_bam_servo", "duck_bam_reset_buffers", "duck_bam_observe", "duck_ppo_loss_scratch",
                     "duck_ppo_loss"):
            getattr(lib, name).restype = I
        _lib = lib
    return _lib


def _raise(status):
    if status != 0:
        raise RuntimeError(library().duck_last_error().decode())


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


class CudaBatch:
    """Batched AVBD environments on one GPU (drop-in for ``_duck_cuda.CudaBatch``)."""

    def __init__(self, model, num_envs, dt=0.001, iterations=200, device=0, fp64=False,
                 specialized=False, shared_memory=False, max_pairs=32):
        """``max_pairs`` (extension): largest accepted number of body-collision
        pairs; 32 is the reference's limit, up to 128 accepted."""
        lib = library()
        self.device = torch.device("cuda", int(device))
        handle = ctypes.c_void_p()
        options = (ctypes.c_int * 1)(int(max_pairs))
        with torch.cuda.device(self.device):
            status = lib.duck_batch_create_ex(str(model).encode(), int(num_envs), float(dt),
                                              int(iterations), int(device), int(bool(fp64)),
                                              int(bool(specialized)), int(bool(shared_memory)),
                                              ctypes.cast(options, ctypes.c_void_p),
                                              _stream(self.device), ctypes.byref(handle))
        _raise(status)
        self._h = handle.value
        info = (ctypes.c_int32 * 10)()
        lib.duck_batch_info(self._h, info)
        (self.num_envs, self.num_bodies, self.num_joints, self.contact_bound, self.record_length,
         _, _, self.envs_per_block, self.lanes_per_env, self.shared_bytes_per_block) = list(info)
        self.dtype = torch.float64 if fp64 else torch.float32
        self._names = [lib.duck_batch_joint_name(self._h, i).decode() for i in range(self.num_joints)]
        counts = (ctypes.c_int32 * 4)()
        _raise(lib.duck_batch_model_counts(self._h, counts))
        self.num_shapes, self.num_pairs = int(counts[2]), int(counts[3])

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and _lib is not None:
            _lib.duck_batch_destroy(h)
            self._h = None

    # ------------------------------------------------------------------ checks
    def _check(self, t, shape, dtype=None):
        dtype = dtype or self.dtype
        if not (isinstance(t, torch.Tensor) and t.is_cuda and t.device == self.device
                and t.dtype == dtype and t.is_contiguous() and tuple(t.shape) == tuple(shape)):
            raise RuntimeError("Invalid CUDA tensor device/dtype/shape/contiguity")
        t.record_stream(torch.cuda.current_stream(self.device))
        return ctypes.c_void_p(t.data_ptr())

    def _empty(self, *shape):
        return torch.empty(shape, device=self.device, dtype=self.dtype)

    # ------------------------------------------------------------------ API
    def reset(self, mask, q, root):
        E, J = self.num_envs, self.num_joints
        with torch.cuda.device(self.device):
            m = self._check(mask, (E,), torch.bool)
            qp = self._check(q, (E, J))
            rp = self._check(root, (E, 6))
            _raise(library().duck_batch_reset(self._h, m, qp, rp, _stream(self.device)))

    def step(self, target, forces, substeps, kp, limit):
        E, J = self.num_envs, self.num_joints
        with torch.cuda.device(self.device):
            tp = self._check(target, (E, J))
            fp = self._check(forces, (E, 3))
            _raise(library().duck_batch_step(self._h, tp, fp, int(substeps), float(kp), float(limit),
                                             _stream(self.device)))

    def step_motor(self, motor, forces):
        E, J = self.num_envs, self.num_joints
        with torch.cuda.device(self.device):
            mp = self._check(motor, (E, J, 3))
            fp = self._check(forces, (E, 3))
            _raise(library().duck_batch_step_motor(self._h, mp, fp, _stream(self.device)))

    def state(self):
        E, B, J = self.num_envs, self.num_bodies, self.num_joints
        with torch.cuda.device(self.device):
            b, j, d = self._empty(E, B, 13), self._empty(E, J, 2), self._empty(E, 6)
            _raise(library().duck_batch_state(self._h, b.data_ptr(), j.data_ptr(), d.data_ptr(),
                                              _stream(self.device)))
        return [b, j, d]

    def contact_forces(self, ground_only=False):
        with torch.cuda.device(self.device):
            out = self._empty(self.num_envs, self.num_bodies, 3)
            _raise(library().duck_batch_contact_forces(self._h, out.data_ptr(), int(bool(ground_only)),
                                                       _stream(self.device)))
        return out

    def self_contact_stats(self):
        with torch.cuda.device(self.device):
            out = self._empty(self.num_envs, 2)
            _raise(library().duck_batch_self_contact_stats(self._h, out.data_ptr(), _stream(self.device)))
        return out

    def contact_counts(self):
        with torch.cuda.device(self.device):
            out = self._empty(self.num_envs, 2)
            _raise(library().duck_batch_contact_counts(self._h, out.data_ptr(), _stream(self.device)))
        return out

    def generalized_loads(self, offset):
        with torch.cuda.device(self.device):
            op = self._check(offset, (self.num_envs, 3))
            out = self._empty(self.num_envs, self.num_joints, 3)
            _raise(library().duck_batch_generalized_loads(self._h, op, out.data_ptr(),
                                                          _stream(self.device)))
        return out

    def reference(self, target, forces, substeps, kp, limit):
        J = self.num_joints
        for t, shape in ((target, (J,)), (forces, (3,))):
            if not (isinstance(t, torch.Tensor) and t.device.type == "cpu" and t.is_contiguous()
                    and t.dtype == self.dtype and tuple(t.shape) == shape):
                raise RuntimeError("Invalid CPU reference target")
        if substeps <= 0:
            raise RuntimeError("Invalid CPU reference inputs")
        b = torch.empty(self.num_bodies, 13, dtype=self.dtype)
        j = torch.empty(J, 2, dtype=self.dtype)
        d = torch.empty(6, dtype=self.dtype)
        with torch.cuda.device(self.device):
            _raise(library().duck_batch_reference(self._h, target.data_ptr(), forces.data_ptr(),
                                                  int(substeps), float(kp), float(limit),
                                                  b.data_ptr(), j.data_ptr(), d.data_ptr()))
        return [b, j, d]

    @property
    def joint_names(self):
        return list(self._names)

    # ------------------------------------------------------------------ extras
    def export_records(self, first=0, count=None):
        """Portable per-env records [count, record_length] (see oracle/avbd_oracle.cpp)."""
        count = self.num_envs - first if count is None else count
        with torch.cuda.device(self.device):
            out = torch.empty(count, self.record_length, device=self.device, dtype=self.dtype)
            _raise(library().duck_batch_export(self._h, first, count, out.data_ptr(), _stream(self.device)))
        return out

    def import_records(self, records, first=0):
        count = records.shape[0]
        with torch.cuda.device(self.device):
            rp = self._check(records, (count, self.record_length))
            _raise(library().duck_batch_import(self._h, first, count, rp, _stream(self.device)))

    def contact_keys(self, env):
        """int32 [n,5] rows (body, shape, feature, other, otherShape) of one env."""
        import numpy as np

        cap = max(self.contact_bound, 1)
        keys = np.zeros((cap, 5), np.int32)
        count = ctypes.c_int()
        with torch.cuda.device(self.device):
            _raise(library().duck_batch_contact_keys(self._h, int(env), keys.ctypes.data_as(ctypes.c_void_p),
                                                     cap, ctypes.byref(count), _stream(self.device)))
        return keys[:count.value].copy()

    def set_parameters(self, mass=None, inertia=None, friction=None):
        """Per-environment physical parameters (extension; the reference shares
        one model): body masses [E,B], principal inertias [E,B,3], ground
        friction per shape [E,S], CUDA tensors of the batch dtype; None keeps
        or restores the model's values.  Invalid values set the environment's
        failure flag."""
        E, B = self.num_envs, self.num_bodies
        with torch.cuda.device(self.device):
            mp = self._check(mass, (E, B)) if mass is not None else None
            ip = self._check(inertia, (E, B, 3)) if inertia is not None else None
            fp = self._check(friction, (E, self.num_shapes)) if friction is not None else None
            _raise(library().duck_batch_set_parameters(self._h, mp, ip, fp, _stream(self.device)))

    @property
    def launches(self):
        """Kernel launches issued by this batch so far."""
        return int(library().duck_batch_launches(self._h))


def fp32_peak_tflops(device=0, iterations=1 << 16):
    """Measured FP32 FMA throughput of ``device`` (TFLOP/s, 2 flops per FMA)."""
    out = ctypes.c_double()
    with torch.cuda.device(device):
        _raise(library().duck_fp32_peak(int(device), int(iterations), ctypes.byref(out),
                                        _stream(torch.device("cuda", device))))
    return out.value
