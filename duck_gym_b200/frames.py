"""Quaternion frame helpers of the tensor environments, written with torch
ops: the reference's ``multiply`` and ``inverse_rotate``
(python/duck_gym/tensor_env.py:9-23), used by ``TensorEnv.state``."""

import torch


def multiply(a, b):
    """Hamilton product of [..., 4] (w, x, y, z) quaternions."""
    w = a[..., :1] * b[..., :1] - (a[..., 1:] * b[..., 1:]).sum(-1, keepdim=True)
    xyz = a[..., :1] * b[..., 1:] + b[..., :1] * a[..., 1:] + torch.linalg.cross(a[..., 1:], b[..., 1:])
    return torch.cat((w, xyz), dim=-1)


def inverse_rotate(q, v):
    """Rotate v by the inverse of unit quaternion q."""
    t = 2 * torch.linalg.cross(-q[..., 1:], v)
    return v + q[..., :1] * t + torch.linalg.cross(-q[..., 1:], t)
