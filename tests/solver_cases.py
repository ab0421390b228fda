"""Scenes for the independent check against the reference's FP64 solver
(``duck_sim``, src/main.cpp + src/solver.cpp), restated as DUCK_MODEL files.

The reference builds these scenes with MuJoCo (scripts/validate_cpu.py:21-38,
scripts/validate_cuda.py:35-37: free fall, pendulum, motor, joint friction,
joint stiction, joint limit, sphere drop, box at rest, box slide, free
rotation, MicroDuck release).  MuJoCo is not available, so each scene is
written directly in the loader's format (src/solver.cpp:67-174) with the same
bodies, shapes, initial states and applied torques; the MicroDuck release uses
the seeded synthetic biped.  The gates are the reference's
(scripts/validate_cuda.py:116-121): position within 2 mm (fp64) / 10 mm (fp32)
of duck_sim, rotation within 0.05 rad, joint error and penetration within
5 mm, with kp = 0, dt 1 ms and 200 iterations.
"""

import math

WORLD = "world 0 0 0 0 0 0 0 1 0 0 0 0 0 0 0 0 0"


def _fmt(*values):
    return " ".join(format(float(v), ".17g") if not isinstance(v, str) else v for v in values)


def _body(name, mass, inertia, x, q=(1, 0, 0, 0), v=(0, 0, 0), w=(0, 0, 0)):
    return _fmt(name, mass, *inertia, *x, *q, *v, *w)


def _box_inertia(mass, half):
    a, b, c = (2 * h for h in half)
    return (mass * (b * b + c * c) / 12, mass * (a * a + c * c) / 12, mass * (a * a + b * b) / 12)


def _hinge(a, b, ra, rb, axis, tangent, limited=0, lo=0, hi=0, damping=0, armature=0, friction=0, torque=0):
    return _fmt("hinge", int(a), int(b), *ra, *rb, *axis, *axis, *tangent, *tangent, int(limited), lo, hi,
                damping, armature, friction, torque, 0, 0, 0)


def _shape(body, kind, size, friction=1.0):
    return f"{body} {kind} 0 0 0 1 0 0 0 " + _fmt(*size, friction) + " 0"


def _model(gravity, ground, bodies, joints=(), shapes=()):
    head = f"DUCK_MODEL 1 {len(bodies) + 1} {len(joints)} {len(shapes)}"
    return "\n".join([head, _fmt(*gravity, int(ground)), WORLD, *bodies, *joints, *shapes]) + "\n"


G = (0, 0, -9.81)
BALL = (1.0, (0.001, 0.001, 0.001))          # 5 cm sphere, 1 kg: 2/5 m r^2
ROTOR_HALF = (0.1, 0.05, 0.02)


def _rotor(limited=0, lo=0, hi=0, damping=0.01, armature=0.002, friction=0.0, torque=0.01):
    body = _body("rotor", 1.0, _box_inertia(1.0, ROTOR_HALF), (0, 0, 0))
    joint = _hinge(0, 1, (0, 0, 0), (0, 0, 0), (0, 0, 1), (1, 0, 0), limited, lo, hi, damping, armature, friction,
                   torque)
    return _model((0, 0, 0), False, [body], [joint], [_shape(1, 1, ROTOR_HALF)])


def _pendulum(angle=0.5, length=0.5):
    half = length / 2
    q = (math.cos(angle / 2), 0.0, math.sin(angle / 2), 0.0)
    x = (-half * math.sin(angle), 0.0, 1.0 - half * math.cos(angle))
    inertia = (length * length / 12 + 0.00045, length * length / 12 + 0.00045, 0.00045)
    body = _body("pendulum", 1.0, inertia, x, q)
    joint = _hinge(0, 1, (0, 0, 1), (0, 0, half), (0, 1, 0), (1, 0, 0))
    return _model(G, False, [body], [joint])


BOX_HALF = (0.1, 0.08, 0.08)
SPIN_HALF = (0.1, 0.07, 0.04)

# name: (model text, duration s)
CASES = {
    "freefall": (_model(G, False, [_body("ball", *BALL, (0, 0, 1))], shapes=[_shape(1, 0, (0.05, 0, 0))]), 0.2),
    "pendulum": (_pendulum(), 0.5),
    "motor": (_rotor(), 0.5),
    "joint_friction": (_rotor(friction=0.0048), 0.5),
    "joint_stiction": (_rotor(friction=0.0048, torque=0.002), 0.5),
    "joint_limit": (_rotor(limited=1, lo=-0.2, hi=0.2, damping=0, armature=0, torque=0.02), 0.5),
    "sphere_drop": (_model(G, True, [_body("ball", *BALL, (0, 0, 1))], shapes=[_shape(1, 0, (0.05, 0, 0))]), 0.8),
    "box_rest": (_model(G, True, [_body("box", 1.0, _box_inertia(1.0, BOX_HALF), (0, 0, 0.0801))],
                        shapes=[_shape(1, 1, BOX_HALF)]), 0.5),
    "box_slide": (_model(G, True, [_body("box", 1.0, _box_inertia(1.0, BOX_HALF), (0, 0, 0.0801), v=(0.5, 0, 0))],
                         shapes=[_shape(1, 1, BOX_HALF)]), 0.5),
    "free_rotation": (_model((0, 0, 0), False, [_body("spinner", 1.0, _box_inertia(1.0, SPIN_HALF), (0, 0, 1),
                                                      w=(1, 2, 3))], shapes=[_shape(1, 1, SPIN_HALF)]), 0.2),
}

POSITION_GATE = {True: 0.002, False: 0.01}   # fp64, fp32
ROTATION_GATE = 0.05
JOINT_GATE = PENETRATION_GATE = 0.005
