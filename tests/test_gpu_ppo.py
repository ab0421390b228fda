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


def test_graphed_update_matches_eager(tmp_path):
    """The update replayed from CUDA graphs takes the same steps as the eager
    update: same minibatch order, same KL schedule, same clipped Adam steps
    (parameters, optimizer state and learning rate restored in place between
    the two runs)."""
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from duck_gym_b200 import biped
    from duck_gym_b200.bam_env import BamEnv
    from duck_gym_b200.ppo import PPO, PPOConfig

    biped.write_bam(tmp_path, seed=0)
    env = BamEnv(tmp_path, num_envs=256, iterations=10, auto_reset=True, reward_enabled=True, seconds=0.1)
    agent = PPO(env, PPOConfig(steps_per_env=8), seed=0)
    agent.rollout()
    agent.update()          # eager: creates the optimizer state
    agent.rollout()
    params = [p for p in agent.policy.parameters()]
    saved_params = [p.detach().clone() for p in params]
    saved_state = [{k: v.clone() for k, v in agent.optimizer.state[p].items()} for p in params]
    saved_lr = agent._lr64.clone()

    def restore():
        with torch.no_grad():
            for p, v, st in zip(params, saved_params, saved_state):
                p.copy_(v)
                for k, t in st.items():
                    agent.optimizer.state[p][k].copy_(t)
            agent._lr64.copy_(saved_lr)
            agent._lr.copy_(saved_lr)

    agent.cfg.graph_update = False
    eager_stats = agent.update(generator=torch.Generator(device="cuda").manual_seed(7))
    eager = [p.detach().clone() for p in params]
    eager_lr = agent.learning_rate
    restore()
    agent.cfg.graph_update = True
    graphed_stats = agent.update(generator=torch.Generator(device="cuda").manual_seed(7))
    assert agent._ugraphs is not None
    for a, b in zip(eager, params):
        torch.testing.assert_close(b.detach(), a, rtol=1e-5, atol=1e-6)
    assert agent.learning_rate == pytest.approx(eager_lr, rel=1e-12)
    for k in eager_stats:
        assert graphed_stats[k] == pytest.approx(eager_stats[k], rel=1e-4, abs=1e-6)


def test_gpu_update_matches_restatement(tmp_path):
    """One GPU rollout and one graphed minibatch step checked against the
    numpy restatement of the published algorithm (oracle/ppo_math.py) on the
    GPU's own buffers: GAE returns and normalised advantages; the surrogate,
    clipped value loss, entropy and KL of the minibatch at the parameters it
    starts from; and the learning rate the adaptive KL schedule sets, against
    the host rule."""
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    import numpy as np

    from duck_gym_b200 import biped
    from duck_gym_b200.bam_env import BamEnv
    from duck_gym_b200.ppo import PPO, PPOConfig, kl_schedule_host
    from oracle import ppo_math

    biped.write_bam(tmp_path, seed=0)
    env = BamEnv(tmp_path, num_envs=256, iterations=10, auto_reset=True, reward_enabled=True, seconds=0.1)
    agent = PPO(env, PPOConfig(steps_per_env=8), seed=0)
    agent.rollout()
    agent.update()          # eager: creates the optimizer state
    agent.rollout()
    s, cfg = agent.storage, agent.cfg
    host = lambda t: t.detach().double().cpu().numpy()
    # GAE on the stored rewards, done masks and values.
    with torch.no_grad():
        last = agent.policy.value(agent.critic_obs)
    returns, adv = ppo_math.gae(host(s.rewards), host(s.dones), host(s.values), host(last), cfg.gamma, cfg.lam)
    adv = (adv - adv.mean()) / (adv.std(ddof=1) + 1e-8)
    np.testing.assert_allclose(host(s.returns), returns, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(host(s.advantages), adv, rtol=1e-4, atol=1e-5)
    assert s.dones.sum() > 0
    # One minibatch of the graphed update.
    agent._prepare_flat()
    n = s.T * s.E
    idx = torch.randperm(n, device="cuda", generator=torch.Generator(device="cuda").manual_seed(3))[: n // 4]
    flat = lambda x: x.reshape(n, *x.shape[2:])[idx]
    with torch.no_grad():
        mu = agent.policy.mean(flat(s.obs))
        value = agent.policy.value(flat(s.critic_obs))
    sigma = np.broadcast_to(host(agent.policy.std), mu.shape)
    want = ppo_math.ppo_terms(host(mu), sigma, host(value), host(flat(s.actions)), host(flat(s.log_prob)),
                              host(flat(s.mu)), host(flat(s.sigma)), host(flat(s.values)), host(flat(s.returns)),
                              host(flat(s.advantages)), cfg.clip)
    lr_before = agent.learning_rate
    agent._idx.copy_(idx)
    agent._run_part(0)
    got = dict(zip(agent.STATS, agent._stats.tolist()))
    for k in agent.STATS:
        assert got[k] == pytest.approx(want[k], rel=2e-4, abs=2e-6), k
    assert agent.learning_rate == pytest.approx(kl_schedule_host(lr_before, got["kl"], cfg.desired_kl), rel=1e-12)


def test_fused_loss_matches_torch_expression():
    """duck_ppo_loss (fused CUDA loss and gradient) against the torch
    expression of ppo_loss on the same minibatch: the loss and its statistics,
    its gradient with respect to the policy means, std and values (all fp32),
    and, through the bf16 MLPs, the gradient of every policy parameter."""
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from duck_gym_b200 import ppo

    torch.manual_seed(5)
    cfg = ppo.PPOConfig(actor_hidden=(64, 32), critic_hidden=(64, 32))
    policy = ppo.ActorCritic(61, 76, 14, cfg).cuda()
    B = 3000
    g = torch.Generator(device="cuda").manual_seed(6)
    r = lambda *s: torch.randn(*s, device="cuda", generator=g)
    obs, cobs = r(B, 61), r(B, 76)
    with torch.no_grad():
        old_mu = policy.mean(obs) + 0.05 * r(B, 14)
    old_sigma = torch.full((B, 14), 0.15, device="cuda") * (1 + 0.1 * r(B, 14)).abs()
    actions = old_mu + old_sigma * r(B, 14)
    old_lp = torch.distributions.Normal(old_mu, old_sigma).log_prob(actions).sum(-1)
    tv, ret, adv = r(B), r(B), r(B)
    # The loss as a function of (mu, std, value): fused against torch.
    with torch.no_grad():
        mu0, v0 = policy.mean(obs), policy.value(cobs)
    grads = []
    for fused in (False, True):
        mu = mu0.clone().requires_grad_(True)
        std = policy.std.detach().clone().requires_grad_(True)
        value = v0.clone().requires_grad_(True)
        if fused:
            loss, stats = ppo.FusedPPOLoss.apply(mu, std, value, actions, old_lp, old_mu, old_sigma, tv, ret, adv,
                                                 cfg.clip, cfg.value_coef, cfg.entropy_coef)
            stats = stats.tolist()
        else:
            d = torch.distributions.Normal(mu, std.expand(B, -1))
            lp, ent = d.log_prob(actions).sum(-1), d.entropy().sum(-1)
            ratio = torch.exp(lp - old_lp)
            surr = torch.max(-adv * ratio, -adv * ratio.clamp(1 - cfg.clip, 1 + cfg.clip)).mean()
            clipped = tv + (value - tv).clamp(-cfg.clip, cfg.clip)
            vl = torch.max((value - ret).square(), (clipped - ret).square()).mean()
            kl = (torch.log(std / old_sigma + 1e-5) + (old_sigma.square() + (old_mu - mu).square())
                  / (2.0 * std.square()) - 0.5).sum(-1).mean()
            loss = surr + cfg.value_coef * vl - cfg.entropy_coef * ent.mean()
            stats = [float(surr), float(vl), float(ent.mean()), float(kl)]
        loss.backward()
        grads.append((float(loss.detach()), stats, mu.grad, std.grad, value.grad))
    (l0, s0, *g0), (l1, s1, *g1) = grads
    assert l1 == pytest.approx(l0, rel=1e-5, abs=1e-6)
    assert s1 == pytest.approx(s0, rel=1e-5, abs=1e-6)
    for a, b in zip(g0, g1):
        torch.testing.assert_close(b, a, rtol=1e-4, atol=1e-9)
    # Through the policy (bf16 MLPs): same parameter gradients up to bf16 rounding.
    pg = []
    for fused in (False, True):
        cfg.fused_loss = fused
        policy.zero_grad()
        loss, _ = ppo.ppo_loss(policy, obs, cobs, actions, old_lp, old_mu, old_sigma, tv, ret, adv, cfg)
        loss.backward()
        pg.append([p.grad.detach().clone() for p in policy.parameters()])
    for a, b in zip(*pg):
        assert float((b - a).norm()) <= 1e-2 * float(a.norm()) + 1e-9
