"""Seeded synthetic MicroDuck-like biped, written as a ``DUCK_MODEL`` text file.

The reference benchmarks the official MicroDuck meshes, which are prepared from
MuJoCo assets (``scripts/prepare_standing.py``, ``scripts/model_io.py:89-272``).
Neither MuJoCo nor the assets exist here, so this module generates a stand-in
with the same topology: world + floating base + 14 hinged links (two legs of
five, neck 2, head 2), joint names and order as the reference's specialized
layout (``src/cuda/extension.cu:228-231``).

Generation rules (seed-driven, numpy ``default_rng(seed)``):

* base: box 0.10 x 0.08 x 0.06 m, mass 0.20 kg;
* every link length ~ U[0.03, 0.08] m; shape type capsule or box with equal
  probability, except the feet (always flat boxes, 1.5x the drawn length) and
  the head (box).  The right leg mirrors the left leg's draws (lengths, shape
  types and masses), so both feet reach the ground at HOME;
* link masses ~ U[0.02, 0.15] kg, then rescaled so that the 14 links weigh
  0.50 kg together (0.70 kg total).  The draw alone averages 1.19 kg, which
  contradicts the requested ~0.7 kg total; rescaling keeps the relative spread;
* shapes cover the middle 70 % of each link so that non-adjacent links do not
  touch at rest (relevant once self-contact pairs are enabled);
* the hip yaw and hip roll links are horizontal brackets (their length runs
  along x, the next joint sits 12 mm lower), which keeps the stance short and
  wide enough (hips at y = +-45 mm, feet 50 mm wide) to stand under PD control;
* HOME is a mild crouch; the robot is placed with its lowest collision point
  0.1 mm above the ground, like ``scripts/prepare_standing.py:79-81``.

The file layout follows the reference loader ``src/solver.cpp:67-174``
(version 1: ground only; version 2: per-shape ground flag + collision pairs).
"""

from __future__ import annotations

import json
import math
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

JOINT_NAMES = (
    "left_hip_yaw", "left_hip_roll", "left_hip_pitch", "left_knee", "left_ankle",
    "neck_pitch", "head_pitch", "head_yaw", "head_roll",
    "right_hip_yaw", "right_hip_roll", "right_hip_pitch", "right_knee", "right_ankle",
)

_AXES = {"yaw": (0.0, 0.0, 1.0), "roll": (1.0, 0.0, 0.0), "pitch": (0.0, 1.0, 0.0)}
_LEG = (("hip_yaw", "yaw"), ("hip_roll", "roll"), ("hip_pitch", "pitch"), ("knee", "pitch"),
        ("ankle", "pitch"))
_HEAD = (("neck_pitch", "pitch"), ("head_pitch", "pitch"), ("head_yaw", "yaw"),
         ("head_roll", "roll"))

HOME = {
    "hip_yaw": 0.0, "hip_roll": 0.0, "hip_pitch": -0.25, "knee": 0.5, "ankle": -0.25,
    "neck_pitch": 0.2, "head_pitch": -0.2, "head_yaw": 0.0, "head_roll": 0.0,
}
LIMITS = {
    "hip_yaw": (-0.6, 0.6), "hip_roll": (-0.5, 0.5), "hip_pitch": (-1.2, 1.0),
    "knee": (-0.3, 1.6), "ankle": (-1.0, 1.0), "neck_pitch": (-0.8, 0.8),
    "head_pitch": (-0.8, 0.8), "head_yaw": (-0.8, 0.8), "head_roll": (-0.8, 0.8),
}

BASE_MASS = 0.20
LINK_MASS_TOTAL = 0.50
JOINT_DAMPING = 0.02
JOINT_ARMATURE = 0.0005
JOINT_FRICTIONLOSS = 0.002
SHAPE_FRICTION = 0.8
# Nominal PD gains of the synthetic biped for the PD-controlled configurations.
# At dt = 5 ms with 10 AVBD iterations a 4 N m/rad spring lets the knees sag
# until the robot topples; 20 N m/rad with a 2 N m cap holds HOME for most
# seeds and fixed target perturbations of 0.05 rad.
KP = 20.0
TORQUE_LIMIT = 2.0


def _qmul(a, b):
    aw, ax, ay, az = a
    bw, bx, by, bz = b
    return np.array([
        aw * bw - ax * bx - ay * by - az * bz,
        aw * bx + ax * bw + ay * bz - az * by,
        aw * by - ax * bz + ay * bw + az * bx,
        aw * bz + ax * by - ay * bx + az * bw,
    ])


def _rot(q, v):
    u = np.asarray(q[1:])
    v = np.asarray(v, dtype=float)
    return v + 2.0 * np.cross(u, np.cross(u, v) + q[0] * v)


def _axis_quat(axis, angle):
    axis = np.asarray(axis, dtype=float)
    return np.r_[math.cos(angle / 2), math.sin(angle / 2) * axis]


@dataclass
class _Link:
    name: str
    parent: int
    axis: np.ndarray
    anchor: np.ndarray          # joint anchor, world frame, zero pose
    com: np.ndarray             # centre of mass, world frame, zero pose
    kind: int                   # 1 box, 2 capsule
    size: np.ndarray            # duck shape size triple
    shape_q: np.ndarray         # shape frame in the body frame (wxyz)
    mass: float = 0.0
    inertia: np.ndarray = field(default_factory=lambda: np.zeros(3))
    lo: float = 0.0
    hi: float = 0.0
    home: float = 0.0


def _inertia(kind, size, mass, shape_q=(1.0, 0.0, 0.0, 0.0)):
    """Diagonal inertia in the body frame; capsules run along the shape's z,
    which is the body's z or (for brackets) the body's x."""
    if kind == 1:
        a, b, c = size
        return mass / 3.0 * np.array([b * b + c * c, a * a + c * c, a * a + b * b])
    r, h = size[0], size[1]
    length = 2 * (h + r)
    perp, along = mass * (3 * r * r + length * length) / 12.0, mass * r * r / 2.0
    if abs(shape_q[0] - 1.0) > 1e-12:
        return np.array([along, perp, perp])
    return np.array([perp, perp, along])


def _shape_points(kind, size):
    """Local support points used only to place the robot above the ground."""
    if kind == 1:
        return [np.array([sx * size[0], sy * size[1], sz * size[2]])
                for sx in (-1, 1) for sy in (-1, 1) for sz in (-1, 1)]
    return [np.array([0.0, 0.0, s * size[1]]) for s in (-1, 1)]


def generate(seed: int = 0, self_contacts: bool = False):
    """Return (model text, metadata dict) for the seeded biped."""
    rng = np.random.default_rng(seed)
    base_half = np.array([0.05, 0.04, 0.03])
    links: list[_Link] = []

    draws = {}

    def chain(prefix, spec, start, parent_body, direction, mirror=None):
        anchor = np.array(start, dtype=float)
        parent = parent_body
        for i, (joint, axis_name) in enumerate(spec):
            foot = joint == "ankle"
            head = joint == "head_roll"
            bracket = joint in ("hip_yaw", "hip_roll")
            if mirror is not None:
                length, coin = draws[mirror + joint]
            else:
                length, coin = float(rng.uniform(0.03, 0.08)), float(rng.uniform())
                draws[prefix + joint] = (length, coin)
            shape_q = np.array([1.0, 0.0, 0.0, 0.0])
            step = direction * length
            if foot or head:
                kind = 1
            else:
                kind = 1 if coin < 0.5 else 2
            if foot:
                size = np.array([0.75 * length, 0.025, 0.005])
                com = anchor + np.array([0.3 * length / 2, 0.0, -0.009])
            elif bracket:
                step = -0.012
                com = anchor + np.array([0.0, 0.0, -0.006])
                if kind == 1:
                    size = np.array([0.7 * length / 2, 0.012, 0.005])
                else:
                    radius = min(0.006, 0.7 * length / 4)
                    size = np.array([radius, max(0.7 * length / 2 - radius, 1e-3), 0.0])
                    shape_q = _axis_quat((0.0, 1.0, 0.0), math.pi / 2)
            elif head:
                size = np.array([0.03, 0.035, 0.7 * length / 2])
                com = anchor + np.array([0.0, 0.0, direction * length / 2])
            elif kind == 1:
                size = np.array([0.012, 0.012, 0.7 * length / 2])
                com = anchor + np.array([0.0, 0.0, direction * length / 2])
            else:
                radius = min(0.01, 0.7 * length / 4)
                size = np.array([radius, max(0.7 * length / 2 - radius, 1e-3), 0.0])
                com = anchor + np.array([0.0, 0.0, direction * length / 2])
            name = prefix + joint
            key = joint if joint in HOME else joint
            links.append(_Link(name, parent, np.array(_AXES[axis_name]), anchor.copy(), com,
                               kind, size, shape_q, lo=LIMITS[key][0], hi=LIMITS[key][1],
                               home=HOME[key]))
            parent = len(links) + 1
            anchor = anchor + np.array([0.0, 0.0, step])

    base_com = np.zeros(3)
    chain("left_", _LEG, [0.0, 0.045, -base_half[2]], 1, -1.0)
    chain("", _HEAD, [0.0, 0.0, base_half[2]], 1, 1.0)
    chain("right_", _LEG, [0.0, -0.045, -base_half[2]], 1, -1.0, mirror="left_")
    assert tuple(l.name for l in links) == JOINT_NAMES

    raw = rng.uniform(0.02, 0.15, size=len(links))
    raw[9:14] = raw[0:5]
    masses = raw * (LINK_MASS_TOTAL / raw.sum())
    for link, m in zip(links, masses):
        link.mass = float(m)
        link.inertia = _inertia(link.kind, link.size, link.mass, link.shape_q)

    # Zero-pose bodies: 0 world, 1 base, 2.. links; every body frame is world
    # aligned at the zero pose, so axes/tangents/anchors are frame constants.
    com0 = [np.zeros(3), base_com] + [l.com for l in links]
    # Forward kinematics to HOME.
    quats = [np.array([1.0, 0, 0, 0]), np.array([1.0, 0, 0, 0])]
    pos = [np.zeros(3), base_com.copy()]
    for link in links:
        qa, xa = quats[link.parent], pos[link.parent]
        ra = link.anchor - com0[link.parent]
        rb = link.anchor - link.com
        qb = _qmul(qa, _axis_quat(link.axis, link.home))
        p = xa + _rot(qa, ra)
        quats.append(qb)
        pos.append(p - _rot(qb, rb))

    identity = np.array([1.0, 0.0, 0.0, 0.0])
    shapes = [(1, 1, np.zeros(3), identity, base_half)] + [
        (i + 2, l.kind, np.zeros(3), l.shape_q, l.size) for i, l in enumerate(links)]
    lowest = math.inf
    for body, kind, centre, shape_q, size in shapes:
        for p in _shape_points(kind, size):
            world = pos[body] + _rot(quats[body], centre + _rot(shape_q, p))
            z = world[2] - (size[0] if kind == 2 else 0.0)
            lowest = min(lowest, z)
    lift = 0.0001 - lowest
    pos = [p if i == 0 else p + np.array([0, 0, lift]) for i, p in enumerate(pos)]

    def fmt(values):
        return " ".join(v if isinstance(v, str) else (str(v) if isinstance(v, (int, np.integer))
                                                     else format(float(v), ".17g"))
                        for v in values)

    lines = [f"DUCK_MODEL {2 if self_contacts else 1} {len(pos)} {len(links)} {len(shapes)}",
             fmt([0.0, 0.0, -9.81, 1])]
    lines.append(fmt(["world", 0.0, 0, 0, 0, 0, 0, 0, 1, 0, 0, 0, 0, 0, 0, 0, 0, 0]))
    base_inertia = _inertia(1, base_half, BASE_MASS)
    bodies = [("base", BASE_MASS, base_inertia)] + [(l.name + "_link", l.mass, l.inertia)
                                                    for l in links]
    for i, (name, mass, inertia) in enumerate(bodies, start=1):
        lines.append(fmt([name, mass, *inertia, *pos[i], *quats[i], 0, 0, 0, 0, 0, 0]))
    for i, link in enumerate(links):
        a, b = link.parent, i + 2
        t = np.cross(link.axis, [1, 0, 0] if abs(link.axis[0]) < 0.8 else [0, 1, 0])
        t = t / np.linalg.norm(t)
        ra = link.anchor - com0[a]
        rb = link.anchor - link.com
        lines.append(fmt([link.name, a, b, *ra, *rb, *link.axis, *link.axis, *t, *t, 1,
                          link.lo, link.hi, JOINT_DAMPING, JOINT_ARMATURE, JOINT_FRICTIONLOSS,
                          0.0, 0.0, 0.0, 0.0]))
    for body, kind, centre, shape_q, size in shapes:
        row = [body, kind, *centre, *shape_q, *size, SHAPE_FRICTION, 0]
        if self_contacts:
            row.append(1)
        lines.append(fmt(row))
    if self_contacts:
        parent = {i + 2: l.parent for i, l in enumerate(links)}
        pairs = []
        for sa in range(len(shapes)):
            for sb in range(sa + 1, len(shapes)):
                ba, bb = shapes[sa][0], shapes[sb][0]
                if ba == bb or parent.get(ba) == bb or parent.get(bb) == ba:
                    continue
                pairs.append((sa, sb, SHAPE_FRICTION))
        lines.append(str(len(pairs)))
        lines += [fmt([a, b, mu]) for a, b, mu in pairs]
    text = "\n".join(lines) + "\n"
    meta = dict(
        joint_names=list(JOINT_NAMES),
        home=[l.home for l in links],
        lower=[l.lo for l in links],
        upper=[l.hi for l in links],
        root_iquat=[1.0, 0.0, 0.0, 0.0],
        root_height=float(pos[1][2]),
        mass=float(BASE_MASS + sum(l.mass for l in links)),
        kp=KP,
        torque_limit=TORQUE_LIMIT,
        seed=seed,
        self_contacts=self_contacts,
        generator="duck_gym_b200.biped",
    )
    return text, meta


# Synthetic stand-in for the pinned BAM XL330/m6 parameter file (the reference
# loads it from the third-party ``bam`` package, bam/params/xl330/m6.json at
# commit 62bd8ce, which is not available here).  The keys are the ones the
# reference actuator reads (python/duck_gym/actuator.py:46-73).  The values are
# chosen, not fitted: with vin 7 V and kp_fw 993 the servo behaves as the BAM
# motor model of the self-contact configuration -- proportional gain
# kt vin kp_fw g / R = 4.0 N m/rad (g = 4096 / (2 pi) / (256 * 885) counts per
# radian over the firmware scale), back-EMF damping kt^2 / R = 0.1 N m s/rad,
# torque limit 0.5 N m -- plus load- and speed-dependent dry friction.
BAM_PARAMETERS = dict(
    kt=0.5, R=2.5, friction_base=0.004, friction_stribeck=0.003, load_friction_external=0.02,
    load_friction_motor=0.015, load_friction_external_stribeck=0.01, load_friction_motor_stribeck=0.008,
    load_friction_external_quad=0.04, load_friction_motor_quad=0.03, dtheta_stribeck=0.2, alpha=1.4,
    friction_viscous=0.006,
)
BAM_SUPPLY = dict(kp_fw=993.0, vin=7.0, vin_drop_gain=0.1, vin_min=6.0, force_limit=0.5)
FOOT_JOINTS = ("left_ankle", "right_ankle")


def bam_config(text: str, meta: dict, physics_dt: float = 0.005, decimation: int = 4,
               delay_lag_steps=(1, 3), root_com_offset=(0.004, 0.0, -0.006)) -> dict:
    """The ``config.json`` of a BAM bundle for a generated biped, with the keys
    the reference ``BamEnv`` reads (python/duck_gym/bam_env.py:33-133, written
    by scripts/prepare_official_model.py:109-145 from MuJoCo there): foot
    bodies with their collision corners and sole sites in body coordinates,
    HOME as ``default_qpos[7:]``, and the synthetic servo parameters above."""
    lines = text.splitlines()
    n_bodies = int(lines[0].split()[2])
    n_joints = int(lines[0].split()[3])
    shape_rows = [line.split() for line in lines[2 + n_bodies + n_joints:2 + n_bodies + n_joints + int(lines[0].split()[4])]]
    feet = []
    for joint in FOOT_JOINTS:
        body = 2 + JOINT_NAMES.index(joint)
        row = next(r for r in shape_rows if int(r[0]) == body)
        hx, hy, hz = (float(v) for v in row[9:12])
        cx, cy, cz = (float(v) for v in row[2:5])
        corners = [[cx + sx * hx, cy + sy * hy, cz + sz * hz] for sx in (-1, 1) for sy in (-1, 1) for sz in (-1, 1)]
        feet.append(dict(body=body, points=corners, site=[cx, cy, cz - hz]))
    base = lines[3].split()
    return dict(
        scope="Synthetic biped bundle (duck_gym_b200.biped); BAM parameters are chosen stand-ins",
        physics_dt=physics_dt,
        decimation=decimation,
        default_qpos=[float(v) for v in base[5:8]] + [float(v) for v in base[8:12]] + list(meta["home"]),
        root_com_offset=list(root_com_offset),
        root_principal_quat=list(meta["root_iquat"]),
        feet=feet,
        masses=[float(line.split()[1]) for line in lines[2:2 + n_bodies]],
        joint_names=list(meta["joint_names"]),
        parameters=dict(BAM_PARAMETERS),
        delay_lag_steps=list(delay_lag_steps),
        **BAM_SUPPLY,
    )


def write_bam(directory, seed: int = 0, self_contacts: bool = False, **kwargs):
    """Write a BAM bundle (``model.duck`` + ``config.json`` + ``metadata.json``)
    for the seeded biped; return the directory."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    text, meta = generate(seed, self_contacts)
    (directory / "model.duck").write_text(text)
    (directory / "metadata.json").write_text(json.dumps(meta, indent=2) + "\n")
    (directory / "config.json").write_text(json.dumps(bam_config(text, meta, **kwargs), indent=2) + "\n")
    return directory


def gait_record(text: str, meta: dict, samples: int = 32, period: float = 0.8, lift: float = 0.008,
                speed: float = 0.05) -> dict:
    """A synthetic ``gait.npz`` record with the keys the reference's tensor
    env reads (python/duck_gym/tensor_env.py:152-171; written from MuJoCo
    inverse kinematics by scripts/prepare_gait.py:120-131 there):
    ``targets`` [4 directions (+x, -x, +y, -y), samples, J] -- HOME plus a
    stepping cycle (hip pitch / roll swing and knee lift, legs half a period
    apart) -- ``foot_collision_points`` [2, 8, 3] (the foot boxes' corners in
    body coordinates), ``foot_bodies`` [2], ``period``, ``lift``, ``speed``."""
    home = np.asarray(meta["home"], dtype=float)
    names = list(meta["joint_names"])
    phase = 2 * np.pi * np.arange(samples) / samples
    table = np.repeat(home[None, None, :], 4, axis=0).repeat(samples, axis=1)
    for d, (axis, sign) in enumerate(((0, 1), (0, -1), (1, 1), (1, -1))):
        for side, shift in (("left_", 0.0), ("right_", np.pi)):
            swing = np.sin(phase + shift)
            knee = np.clip(np.sin(phase + shift), 0, None)
            j = names.index(side + ("hip_pitch" if axis == 0 else "hip_roll"))
            table[d, :, j] += -sign * 0.15 * swing if axis == 0 else sign * 0.08 * swing
            table[d, :, names.index(side + "knee")] += 0.3 * knee
            table[d, :, names.index(side + "ankle")] -= 0.15 * knee
    cfg = bam_config(text, meta)
    feet = cfg["feet"]
    return dict(targets=table, foot_collision_points=np.array([f["points"] for f in feet]),
                foot_bodies=np.array([f["body"] for f in feet]), period=period, lift=lift, speed=speed)


def write_gait(directory, seed: int = 0, **kwargs):
    """Write ``gait.npz`` next to the seeded biped's model and metadata."""
    directory = Path(directory)
    text, meta = generate(seed)
    np.savez_compressed(directory / "gait.npz", **gait_record(text, meta, **kwargs))
    return directory / "gait.npz"


def with_parameters(text: str, mass=None, inertia=None, friction=None) -> str:
    """The model text with one environment's physical parameters substituted:
    body masses [B], principal inertias [B,3] and shape frictions [S] (None
    keeps the model's).  Values are written with 17 significant digits, so a
    float32 value read back is the same float32 -- this is how the per-env
    parameters of ``CudaBatch.set_parameters`` are restated as model files for
    the CPU oracle."""
    lines = text.splitlines()
    head = lines[0].split()
    nb, nj, ns = int(head[2]), int(head[3]), int(head[4])

    def fmt(v):
        return format(float(v), ".17g")

    for b in range(nb):
        row = lines[2 + b].split()
        if float(row[1]) > 0:
            if mass is not None:
                row[1] = fmt(mass[b])
            if inertia is not None:
                row[2:5] = [fmt(v) for v in inertia[b]]
        lines[2 + b] = " ".join(row)
    for k in range(ns):
        at = 2 + nb + nj + k
        row = lines[at].split()
        if friction is not None:
            row[12] = fmt(friction[k])
        lines[at] = " ".join(row)
    return "\n".join(lines) + "\n"


def write(directory, seed: int = 0, self_contacts: bool = False, name: str = "microduck.duck"):
    """Write ``<directory>/<name>`` and ``metadata.json``; return the model path."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    text, meta = generate(seed, self_contacts)
    path = directory / name
    path.write_text(text)
    (directory / "metadata.json").write_text(json.dumps(meta, indent=2) + "\n")
    return path
