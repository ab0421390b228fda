"""CPU: PPO (duck_gym_b200/ppo.py) against the numpy restatement of the
published algorithm (oracle/ppo_math.py), a learning sanity check on a toy
environment, and the multi-rank gradient all-reduce with two gloo ranks."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from duck_gym_b200 import ppo
from oracle import ppo_math


def test_gae_matches_restatement():
    rng = np.random.default_rng(0)
    T, E = 24, 37
    r, v = rng.normal(size=(T, E)), rng.normal(size=(T, E))
    d = (rng.random((T, E)) < 0.1).astype(np.float64)
    last = rng.normal(size=E)
    want_r, want_a = ppo_math.gae(r, d, v, last, 0.99, 0.95)
    got_r, got_a = ppo.gae(*(torch.from_numpy(x) for x in (r, d, v, last)), 0.99, 0.95)
    np.testing.assert_allclose(got_r.numpy(), want_r, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(got_a.numpy(), want_a, rtol=1e-12, atol=1e-12)


def test_ppo_loss_terms_match_restatement():
    torch.manual_seed(1)
    cfg = ppo.PPOConfig(bf16=False, actor_hidden=(16, 8), critic_hidden=(16,))
    policy = ppo.ActorCritic(5, 7, 3, cfg).double()
    with torch.no_grad():
        policy.std.copy_(torch.tensor([0.2, 0.3, 0.25], dtype=torch.float64))
    rng = np.random.default_rng(2)
    n = 64
    t = lambda *s: torch.from_numpy(rng.normal(size=s))
    obs, cobs, actions = t(n, 5), t(n, 7), t(n, 3)
    old_mu, old_sigma = t(n, 3), torch.from_numpy(rng.uniform(0.1, 0.4, (n, 3)))
    old_lp = torch.from_numpy(ppo_math.normal_log_prob(actions.numpy(), old_mu.numpy(), old_sigma.numpy()))
    target_values, returns, advantages = t(n), t(n), t(n)
    loss, info = ppo.ppo_loss(policy, obs, cobs, actions, old_lp, old_mu, old_sigma, target_values, returns,
                              advantages, cfg)
    with torch.no_grad():
        mu = policy.mean(obs).numpy()
        value = policy.value(cobs).numpy()
    sigma = np.broadcast_to(policy.std.detach().numpy(), mu.shape)
    want = ppo_math.ppo_terms(mu, sigma, value, actions.numpy(), old_lp.numpy(), old_mu.numpy(), old_sigma.numpy(),
                              target_values.numpy(), returns.numpy(), advantages.numpy(), cfg.clip)
    for k in ("surrogate", "value", "entropy", "kl"):
        np.testing.assert_allclose(float(info[k]), want[k], rtol=1e-10, atol=1e-12, err_msg=k)
    total = want["surrogate"] + cfg.value_coef * want["value"] - cfg.entropy_coef * want["entropy"]
    np.testing.assert_allclose(float(loss.detach()), total, rtol=1e-10)


class ToyEnv:
    """Reach a per-env target with the action: reward -|a - target|^2,
    episodes of 8 steps (time-outs)."""

    def __init__(self, n=64, seed=0):
        self.num_envs, self.num_actions, self.device = n, 2, torch.device("cpu")
        g = torch.Generator().manual_seed(seed)
        self.target = torch.rand(n, 2, generator=g) - 0.5
        self.t = torch.zeros(n)

    def get_observations(self):
        return torch.cat((self.target, self.t[:, None] / 8), -1)

    def step(self, actions):
        reward = -(actions - self.target).square().sum(-1)
        self.t += 1
        done = self.t >= 8
        self.t[done] = 0
        return self.get_observations(), reward, done, {"time_outs": done.clone()}


def test_ppo_learns_toy_task():
    env = ToyEnv()
    cfg = ppo.PPOConfig(bf16=False, steps_per_env=16, actor_hidden=(32, 32), critic_hidden=(32, 32),
                        learning_rate=3e-3, initial_std=0.5)
    agent = ppo.PPO(env, cfg, device="cpu", seed=0)
    before = agent.storage.rewards.clone()
    history = agent.learn(1)
    first = float(agent.storage.rewards.mean())
    agent.learn(25)
    last = float(agent.storage.rewards.mean())
    assert np.isfinite(history[0]["surrogate"]) and before.abs().sum() == 0
    assert last > first + 0.05, (first, last)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.manual_seed(0)
    cfg = ppo.PPOConfig(bf16=False, actor_hidden=(16, 16), critic_hidden=(16,), bucket_mb=0.0005)
    net = ppo.ActorCritic(4, 4, 2, cfg)
    for p in net.parameters():
        dist.broadcast(p.data, 0)
    reducer = ppo.GradientAllReduce(net.parameters(), cfg.bucket_mb)
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn(32, 4, generator=g)
    loss = net.mean(x).square().sum() + net.value(x).square().sum() + (net.std * x[:, :2]).square().sum()
    loss.backward()
    local = [p.grad.clone() for p in net.parameters()]
    reducer.finish()
    out[rank] = ([p.grad.clone() for p in net.parameters()], local, len(reducer.buckets))
    # Three PPO updates on a toy env per rank stay in sync across ranks: the
    # first averages gradients through the bucket hooks, the others through
    # the flat gradient buffer (one all-reduce with the KL slot).
    env = ToyEnv(n=16, seed=rank)
    agent = ppo.PPO(env, ppo.PPOConfig(bf16=False, steps_per_env=4, actor_hidden=(16,), critic_hidden=(16,)),
                    device="cpu", seed=rank)
    agent.learn(3)
    out[f"params{rank}"] = [p.detach().clone() for p in agent.policy.parameters()]
    out[f"flat{rank}"] = agent._flat_grad is not None and not agent.reducer.enabled
    out[f"lr{rank}"] = agent.learning_rate
    dist.destroy_process_group()


def test_gradient_all_reduce_two_gloo_ranks():
    world = 2
    # The manager's server process is spawned too: forking this
    # multi-threaded process (torch's thread pools) can deadlock the child.
    with mp.get_context("spawn").Manager() as manager:
        out = manager.dict()
        mp.start_processes(_rank, args=(world, _free_port(), out), nprocs=world, start_method="spawn")
        averaged0, local0, buckets = out[0]
        averaged1, local1, _ = out[1]
        assert buckets > 1
        for a0, a1, l0, l1 in zip(averaged0, averaged1, local0, local1):
            torch.testing.assert_close(a0, (l0 + l1) / 2)
            assert torch.equal(a0, a1)
        for p0, p1 in zip(out["params0"], out["params1"]):
            assert torch.equal(p0, p1)
        assert out["flat0"] and out["flat1"] and out["lr0"] == out["lr1"]


def test_device_kl_schedule_matches_host_rule():
    """The learning-rate schedule run on device tensors (no host round trip)
    follows the host rule step for step, including KLs at the thresholds,
    zero, negative and NaN."""
    import random

    from duck_gym_b200.ppo import kl_schedule, kl_schedule_host

    rng = random.Random(0)
    host, dev = 3e-4, torch.tensor(3e-4, dtype=torch.float64)
    for _ in range(3000):
        kl = rng.choice([0.0, -1e-3, float("nan"), 0.02, 0.005, rng.uniform(0.0, 0.05), rng.uniform(0.004, 0.006),
                         rng.uniform(0.019, 0.021)])
        kl32 = torch.tensor(kl, dtype=torch.float32)
        host = kl_schedule_host(host, float(kl32), 0.01)
        dev = kl_schedule(dev, kl32, 0.01)
        assert host == float(dev)
    assert 1e-5 <= host <= 1e-2


def test_flat_update_matches_eager():
    """The flat-gradient minibatch step (the one the GPU replays from CUDA
    graphs) takes the same steps as the eager update on the CPU."""
    def run(flat):
        cfg = ppo.PPOConfig(bf16=False, steps_per_env=8, actor_hidden=(32, 32), critic_hidden=(32,),
                            learning_rate=3e-3, graph_update=flat)
        agent = ppo.PPO(ToyEnv(n=32, seed=3), cfg, device="cpu", seed=0)
        history = agent.learn(4)
        return agent, history

    flat, flat_history = run(True)
    eager, eager_history = run(False)
    assert flat._flat_grad is not None and eager._flat_grad is None
    for a, b in zip(flat.policy.parameters(), eager.policy.parameters()):
        torch.testing.assert_close(a.detach(), b.detach(), rtol=1e-5, atol=1e-6)
    assert flat.learning_rate == pytest.approx(eager.learning_rate, rel=1e-12)
    for h0, h1 in zip(flat_history, eager_history):
        for k in h1:
            assert h0[k] == pytest.approx(h1[k], rel=1e-4, abs=1e-6)
