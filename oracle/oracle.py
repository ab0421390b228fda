"""ctypes binding of the CPU restatement (``libavbd_oracle.so``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s cpu_baseline leg as the checker.  The product package never
imports this module.

``OracleBatch`` mirrors the reference CPU twin ``_duck_reference.CpuBatch32/64``
(``src/cuda/cpu_bindings.cpp:169-184``): numpy arrays in and out, same method
names.  Extra methods expose contact keys, colour counts and the portable
per-env record used to load one state into both the oracle and the GPU batch.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libavbd_oracle.so"
_lib = None


def library():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing; run `make -C oracle` or __graft_entry__.build()")
        lib = ctypes.CDLL(str(LIB_PATH))
        P, I, D = ctypes.c_void_p, ctypes.c_int, ctypes.c_double
        lib.avbd_oracle_last_error.restype = ctypes.c_char_p
        lib.avbd_oracle_create.restype = P
        lib.avbd_oracle_create.argtypes = [ctypes.c_char_p, I, D, I, I, I]
        lib.avbd_oracle_create_ex.restype = P
        lib.avbd_oracle_create_ex.argtypes = [ctypes.c_char_p, I, D, I, I, I, I]
        lib.avbd_oracle_destroy.argtypes = [P]
        lib.avbd_oracle_info.argtypes = [P, P]
        for name, args in {
            "reset": [P, P, P, P],
            "step": [P, P, P, I, D, D, I, I],
            "step_motor": [P, P, P, I],
            "state": [P, P, P, P],
            "contact_forces": [P, P, I],
            "self_contact_stats": [P, P],
            "contact_counts": [P, P],
            "generalized_loads": [P, P, P],
            "contacts": [P, I, P, I],
            "color_count": [P, I],
            "export": [P, I, P],
            "import": [P, I, P],
        }.items():
            fn = getattr(lib, "avbd_oracle_" + name)
            fn.argtypes = args
            fn.restype = I
        lib.avbd_oracle_count_ops.argtypes = [ctypes.c_char_p, I, D, I, P, P, P, P, I, I, D, D, I, P]
        lib.avbd_oracle_count_ops.restype = I
        _lib = lib
    return _lib


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _check(status):
    if status != 0:
        raise ValueError(library().avbd_oracle_last_error().decode())


class OracleBatch:
    """CPU restatement of the AVBD batch; ``capacity`` is the per-env contact
    list size (160 for the reference's generic state, 64 for the compact one)."""

    def __init__(self, model, num_envs, dt, iterations, threads=1, fp64=False, capacity=160,
                 cuda_semantics=True, max_pairs=32):
        lib = library()
        self._h = lib.avbd_oracle_create_ex(str(model).encode(), int(num_envs), float(dt),
                                            int(iterations), int(bool(fp64)), int(capacity), int(max_pairs))
        if not self._h:
            raise ValueError(lib.avbd_oracle_last_error().decode())
        info = np.zeros(6, np.int32)
        lib.avbd_oracle_info(self._h, _ptr(info))
        self.num_envs, self.num_bodies, self.num_joints, self.contact_bound, self.record_length, _ = (
            int(v) for v in info)
        self.dtype = np.float64 if fp64 else np.float32
        self.threads = max(1, min(int(threads), 64))
        self.cuda_semantics = cuda_semantics

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            library().avbd_oracle_destroy(h)
            self._h = None

    def _arr(self, a, shape, dtype=None):
        a = np.ascontiguousarray(a, dtype=dtype or self.dtype)
        if a.shape != tuple(shape):
            raise ValueError(f"Invalid array shape {a.shape}, expected {tuple(shape)}")
        return a

    def reset(self, mask, q, root):
        mask = self._arr(mask, (self.num_envs,), np.bool_)
        q = self._arr(q, (self.num_envs, self.num_joints))
        root = self._arr(root, (self.num_envs, 6))
        _check(library().avbd_oracle_reset(self._h, _ptr(mask), _ptr(q), _ptr(root)))

    def step(self, target, forces, substeps, kp, limit):
        target = self._arr(target, (self.num_envs, self.num_joints))
        forces = self._arr(forces, (self.num_envs, 3))
        _check(library().avbd_oracle_step(self._h, _ptr(target), _ptr(forces), int(substeps),
                                          float(kp), float(limit), self.threads,
                                          int(self.cuda_semantics)))

    def step_motor(self, motor, forces):
        motor = self._arr(motor, (self.num_envs, self.num_joints, 3))
        forces = self._arr(forces, (self.num_envs, 3))
        _check(library().avbd_oracle_step_motor(self._h, _ptr(motor), _ptr(forces), self.threads))

    def state(self):
        b = np.empty((self.num_envs, self.num_bodies, 13), self.dtype)
        j = np.empty((self.num_envs, self.num_joints, 2), self.dtype)
        d = np.empty((self.num_envs, 6), self.dtype)
        _check(library().avbd_oracle_state(self._h, _ptr(b), _ptr(j), _ptr(d)))
        return b, j, d

    def contact_forces(self, ground_only=False):
        out = np.empty((self.num_envs, self.num_bodies, 3), self.dtype)
        _check(library().avbd_oracle_contact_forces(self._h, _ptr(out), int(bool(ground_only))))
        return out

    def self_contact_stats(self):
        out = np.empty((self.num_envs, 2), self.dtype)
        _check(library().avbd_oracle_self_contact_stats(self._h, _ptr(out)))
        return out

    def contact_counts(self):
        out = np.empty((self.num_envs, 2), self.dtype)
        _check(library().avbd_oracle_contact_counts(self._h, _ptr(out)))
        return out

    def generalized_loads(self, offset):
        offset = self._arr(offset, (self.num_envs, 3))
        out = np.empty((self.num_envs, self.num_joints, 3), self.dtype)
        _check(library().avbd_oracle_generalized_loads(self._h, _ptr(offset), _ptr(out)))
        return out

    def contact_keys(self, env):
        """(body, shape, feature, other, otherShape) rows of env's contact list."""
        keys = np.zeros((max(self.contact_bound, 1) + 160, 5), np.int32)
        count = library().avbd_oracle_contacts(self._h, int(env), _ptr(keys), keys.shape[0])
        if count < 0:
            raise ValueError(library().avbd_oracle_last_error().decode())
        return keys[:count].copy()

    def color_count(self, env):
        return int(library().avbd_oracle_color_count(self._h, int(env)))

    def export_env(self, env):
        out = np.zeros(self.record_length, self.dtype)
        _check(library().avbd_oracle_export(self._h, int(env), _ptr(out)))
        return out

    def import_env(self, env, record):
        record = self._arr(record, (self.record_length,))
        _check(library().avbd_oracle_import(self._h, int(env), _ptr(record)))


def count_ops(model, home, targets, forces, dt, iterations, substeps, kp, limit, records=None, threads=1):
    """Count fp32 solver operations of ``targets.shape[0]`` control steps on
    ``targets.shape[1]`` envs, started from ``records`` (float32 portable
    records [n, record length], e.g. exported from a GPU batch) or else from
    HOME, on ``threads`` host threads.  Returns a dict of counts."""
    targets = np.ascontiguousarray(targets, np.float32)
    steps, n, _ = targets.shape
    home = np.ascontiguousarray(home, np.float32)
    forces = np.ascontiguousarray(forces, np.float32)
    if records is not None:
        records = np.ascontiguousarray(records, np.float32)
        if records.ndim != 2 or records.shape[0] != n:
            raise ValueError(f"records must be [{n}, record length], got {records.shape}")
    out = np.zeros(12, np.uint64)
    _check(library().avbd_oracle_count_ops(str(model).encode(), n, float(dt), int(iterations),
                                           _ptr(home), None if records is None else _ptr(records),
                                           _ptr(targets), _ptr(forces), steps,
                                           int(substeps), float(kp), float(limit), int(threads), _ptr(out)))
    names = ("add", "mul", "div", "sqrt", "sin", "cos", "tan", "atan2", "hypot", "remainder",
             "gs_iterations", "physics_steps")
    return dict(zip(names, (int(v) for v in out)))


def reference_module():
    """Import the reference's own CPU solver built under oracle/_ref, or None."""
    import importlib
    import sys

    ref = HERE / "_ref"
    if not any(ref.glob("_duck_reference*.so")):
        return None
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    return importlib.import_module("_duck_reference")
