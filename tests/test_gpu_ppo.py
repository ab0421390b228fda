"""GPU: PPO (duck_gym_b200/ppo.py) rolling out and updating on the fused BAM
environment with the bf16 actor: a short run stays finite, changes the
policy, and the rollout buffers carry the env's rewards and masks."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_ppo_on_bam_env(tmp_path):
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from duck_gym_b200 import biped
    from duck_gym_b200.bam_env import BamEnv
    from duck_gym_b200.ppo import PPO, PPOConfig

    biped.write_bam(tmp_path, seed=0)
    training = dict(command_ranges=[[-0.3, 0.3], [-0.3, 0.3], [-1.0, 1.0]], command_resample_seconds=1.0,
                    reset_joint_noise=0.01, reset_tilt_noise=0.01)
    env = BamEnv(tmp_path, num_envs=256, iterations=10, auto_reset=True, reward_enabled=True, training=training,
                 seconds=0.1)
    assert (env.command[:, 2].abs() <= 1.0).all() and env.command[:, :2].abs().max() <= 0.3
    agent = PPO(env, PPOConfig(steps_per_env=8), seed=0)
    before = torch.cat([p.detach().flatten() for p in agent.policy.parameters()]).clone()
    history = agent.learn(3)
    after = torch.cat([p.detach().flatten() for p in agent.policy.parameters()])
    assert torch.isfinite(after).all() and not torch.equal(before, after)
    assert all(torch.isfinite(torch.tensor(list(h.values()))).all() for h in history)
    s = agent.storage
    assert torch.isfinite(s.rewards).all() and s.dones.sum() > 0
    assert agent.obs.shape == (256, 61) and agent.critic_obs.shape[1] == 76
