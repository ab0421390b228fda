"""CPU: the BAM restatement (oracle/bam_math.py) reproduces the reference
BamEnv bit for bit.  The stepper runs over a fake engine that replays the
engine outputs recorded from the reference run (tests/golden/bam_*.npz), and
must send the recorded motor channels and produce the recorded observations,
rewards, reward terms and masks."""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import bam_math

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = ["bam_head_stability", "bam_heading"]


class ReplayEngine:
    """Returns the recorded outputs of one control step's substeps in order
    and checks the motor channels it is sent."""

    def __init__(self, g, step):
        self.g, self.s = g, step
        self.calls = {k: 0 for k in ("loads", "motor", "state", "forces", "stats")}

    def _next(self, key):
        k = self.calls[key]
        self.calls[key] += 1
        return k

    def generalized_loads(self, offset):
        return torch.from_numpy(self.g["engine_loads"][self.s, self._next("loads")])

    def step_motor(self, motor, forces):
        k = self._next("motor")
        np.testing.assert_array_equal(motor.numpy(), self.g["engine_motor"][self.s, k], err_msg=f"motor {self.s}.{k}")

    def state(self):
        k = self._next("state")
        return tuple(torch.from_numpy(self.g[f"engine_{n}"][self.s, k]) for n in ("bodies", "joints", "diag"))

    def contact_forces(self, ground_only=False):
        return torch.from_numpy(self.g["engine_forces"][self.s, self._next("forces")])

    def self_contact_stats(self):
        return torch.from_numpy(self.g["engine_stats"][self.s, self._next("stats")])


def stepper_for(g):
    settings = json.loads(str(g["settings"]))
    training = json.loads(str(g["training"]))
    cfg_json = json.loads(str(g["config_json"]))
    n = g["actions"].shape[1]
    cfg = bam_math.config_from_bundle(cfg_json, str(g["model"]), n, dt=settings["dt"], step_dt=settings["step_dt"],
                                      max_episode_length=settings["max_episode_length"], training=training)
    st = bam_math.BamStepper(None, cfg, cfg_json, settings["lag"], settings["decimation"], reward_enabled=True,
                             source_iteration=settings["source_iteration"], neutral_head=settings["neutral_head"],
                             head_stability=training.get("head_stability"))
    return st


@pytest.mark.parametrize("case", CASES)
def test_bam_stepper_reproduces_reference_env(case):
    g = np.load(GOLDEN / f"{case}.npz")
    st = stepper_for(g)
    names = json.loads(str(g["term_names"]))
    for s in range(g["actions"].shape[0]):
        buffers = {k[len("before_"):]: torch.from_numpy(g[k][s].copy()) for k in g.files if k.startswith("before_")}
        st.load(buffers, int(g["history_cursor"][s]), int(g["common_step_counter"][s]))
        st.native = ReplayEngine(g, s)
        out = st.step(torch.from_numpy(g["actions"][s]))
        assert st.native.calls["motor"] == st.decimation
        for key, ref in (("done", "done"), ("timeout", "timeouts"), ("failed", "failed"), ("reward", "reward")):
            np.testing.assert_array_equal(out[key].numpy(), g[ref][s], err_msg=f"{case} step {s} {key}")
        np.testing.assert_array_equal(out["obs"]["actor"].numpy(), g["obs_actor"][s])
        np.testing.assert_array_equal(out["obs"]["critic"].numpy(), g["obs_critic"][s])
        assert list(out["terms"]) == names
        terms = torch.stack([out["terms"][n].to(torch.float64) for n in names], -1).numpy()
        np.testing.assert_array_equal(terms, g["terms"][s])


def test_bam_fixtures_cover_failures_timeouts_and_contacts():
    for case in CASES:
        g = np.load(GOLDEN / f"{case}.npz")
        assert g["failed"].sum() > 0 and g["timeouts"].sum() > 0
        assert (np.linalg.norm(g["engine_forces"], axis=-1) > 1e-5).any()
        assert g["obs_actor"].shape[-1] == 61 and g["obs_critic"].shape[-1] in (79, 80)


def test_xl330_restatement_matches_reference_formula_properties():
    """Closed-form checks of the servo restatement: zero error and zero speed
    give zero torque; the duty clamp bounds the torque by the back-EMF band;
    the applied channel is the raw torque clamped to the force limit."""
    p = dict(kt=0.5, R=2.5, friction_base=0.004, friction_stribeck=0.003, load_friction_external=0.02,
             load_friction_motor=0.015, load_friction_external_stribeck=0.01, load_friction_motor_stribeck=0.008,
             load_friction_external_quad=0.04, load_friction_motor_quad=0.03, dtheta_stribeck=0.2, alpha=1.4,
             friction_viscous=0.006)
    z = torch.zeros(2, 3, dtype=torch.float64)
    kw = dict(vin=torch.full((2, 1), 7.0, dtype=torch.float64), vin_drop_gain=0.1, vin_min=6.0, kp_fw=993.0,
              force_limit=0.5)
    motor, raw, supply = bam_math.xl330_m6(z, z, z, z, z, z, p, **kw)
    assert torch.equal(raw, z) and torch.all(supply == 7.0)
    assert torch.allclose(motor[..., 1], torch.full_like(z, 0.004 + 0.003))
    big = torch.full((2, 3), 2.0, dtype=torch.float64)
    motor, raw, _ = bam_math.xl330_m6(big, z, z, z, z, z, p, **kw)
    assert torch.allclose(raw, torch.full_like(z, 0.5 * 7.0 * (2.5 * 1.75 / 7.0) / 2.5))
    assert torch.allclose(motor[..., 0], torch.full_like(z, 0.5))
