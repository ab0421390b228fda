"""PPO rollout and update for the native environments (velocity-command
task, 4096 envs per GPU, actor MLP 61-512-256-128-14 ELU in bf16).

The reference trains with rsl-rl 5's ``OnPolicyRunner`` and ``PPO``
(scripts/train_bam_native.py:14-140) configured from mjlab's
``Mjlab-Velocity-Flat-MicroDuck`` task; neither package is available here.
This module restates rsl-rl's published PPO algorithm in plain torch:

* a Gaussian policy with a scalar (state-independent) std, as the reference
  pins (train_bam_native.py:127-129), actor and critic MLPs with ELU;
* rollouts of ``steps_per_env`` steps; time-out bootstrapping of the reward
  (r += gamma V(s) on time-outs); GAE(gamma, lambda) returns;
* ``epochs`` x ``mini_batches`` updates of the clipped surrogate, the clipped
  value loss and an entropy bonus, with the adaptive KL learning-rate
  schedule and gradient-norm clipping;
* the actor runs under bf16 autocast (tensor cores) in the rollout and the
  update, with fp32 master weights;
* with a process group of several ranks, gradients are averaged across
  ranks by NCCL all-reduces of flat buckets, launched from gradient hooks as
  soon as a bucket is complete (overlapping the rest of the backward pass),
  and the KL used by the schedule is averaged too, so every rank takes the
  same step.
"""

from __future__ import annotations

import math
import warnings
from dataclasses import dataclass

import torch
import torch.distributed as dist
from torch import nn


@dataclass
class PPOConfig:
    steps_per_env: int = 24
    epochs: int = 5
    mini_batches: int = 4
    gamma: float = 0.99
    lam: float = 0.95
    clip: float = 0.2
    value_coef: float = 1.0
    entropy_coef: float = 0.005
    learning_rate: float = 3e-4
    desired_kl: float = 0.01
    max_grad_norm: float = 1.0
    initial_std: float = 0.15
    actor_hidden: tuple = (512, 256, 128)
    critic_hidden: tuple = (512, 256, 128)
    bf16: bool = True
    bucket_mb: float = 0.5
    graph_rollout: bool = True   # replay the rollout's policy step from a CUDA graph (GPU only)
    graph_update: bool = True    # flat-gradient minibatch step after the first update, CUDA graphs on the GPU
    fused_loss: bool = True      # on the GPU: the loss and its gradient in one fused CUDA pass (duck_ppo_loss)


def mlp(sizes):
    layers = []
    for i in range(len(sizes) - 1):
        layers.append(nn.Linear(sizes[i], sizes[i + 1]))
        if i < len(sizes) - 2:
            layers.append(nn.ELU())
    return nn.Sequential(*layers)


class ActorCritic(nn.Module):
    def __init__(self, actor_obs, critic_obs, actions, cfg: PPOConfig):
        super().__init__()
        self.actor = mlp([actor_obs, *cfg.actor_hidden, actions])
        self.critic = mlp([critic_obs, *cfg.critic_hidden, 1])
        self.std = nn.Parameter(torch.full((actions,), float(cfg.initial_std)))
        self.bf16 = cfg.bf16

    def _autocast(self, x):
        # No cast cache: each region casts every weight once anyway, and a
        # cache is not allowed inside a captured CUDA graph.
        return torch.autocast(x.device.type, dtype=torch.bfloat16, enabled=self.bf16, cache_enabled=False)

    def mean(self, obs):
        with self._autocast(obs):
            return self.actor(obs).float()

    def value(self, obs):
        with self._autocast(obs):
            return self.critic(obs).float().squeeze(-1)

    def distribution(self, obs):
        # No argument validation (as rsl-rl's actor-critic sets): its checks
        # read the tensors back on the host, which a CUDA graph cannot hold.
        return torch.distributions.Normal(self.mean(obs), self.std.expand(obs.shape[0], -1), validate_args=False)


class Storage:
    """Rollout buffers [T, E, ...] (rsl-rl RolloutStorage)."""

    def __init__(self, T, E, actor_obs, critic_obs, actions, device):
        z = lambda *s: torch.zeros(*s, device=device)
        self.obs, self.critic_obs = z(T, E, actor_obs), z(T, E, critic_obs)
        self.actions, self.log_prob, self.mu = z(T, E, actions), z(T, E), z(T, E, actions)
        self.sigma = z(T, E, actions)
        self.rewards, self.dones, self.values = z(T, E), z(T, E), z(T, E)
        self.returns, self.advantages = z(T, E), z(T, E)
        self.T, self.E, self.step = T, E, 0


def gae(rewards, dones, values, last_values, gamma, lam):
    """GAE returns and advantages (rsl-rl RolloutStorage.compute_returns):
    delta_t = r_t + gamma (1 - d_t) V_{t+1} - V_t,
    A_t = delta_t + gamma lambda (1 - d_t) A_{t+1},  R_t = A_t + V_t."""
    T = rewards.shape[0]
    returns = torch.empty_like(rewards)
    advantage = torch.zeros_like(last_values)
    for t in reversed(range(T)):
        next_values = last_values if t == T - 1 else values[t + 1]
        live = 1.0 - dones[t]
        delta = rewards[t] + live * gamma * next_values - values[t]
        advantage = delta + live * gamma * lam * advantage
        returns[t] = advantage + values[t]
    return returns, returns - values


class FusedPPOLoss(torch.autograd.Function):
    """The minibatch loss of ppo_loss and its gradient with respect to the
    policy means, std and values in one pass of the library's fused CUDA
    kernels (duck_ppo_loss: two launches, deterministic sums) instead of the
    torch expression's ~80 element-wise kernels and their backward.  Returns
    the loss and the statistics (surrogate, value loss, entropy, kl)."""

    @staticmethod
    def forward(ctx, mu, std, value, actions, old_log_prob, old_mu, old_sigma, target_values, returns, advantages,
                clip, value_coef, entropy_coef):
        import ctypes

        from .cuda_batch import _raise, _stream, library

        lib = library()
        B, A = mu.shape
        args = [t.detach().contiguous().float() for t in (mu, std, value, actions, old_log_prob, old_mu, old_sigma,
                                                           target_values, returns, advantages)]
        scratch = torch.empty(lib.duck_ppo_loss_scratch(B, A), device=mu.device)
        out = torch.empty(5, device=mu.device)
        grad_mu, grad_std, grad_value = torch.empty_like(args[0]), torch.empty_like(args[1]), torch.empty_like(args[2])
        P = lambda t: ctypes.c_void_p(t.data_ptr())
        _raise(lib.duck_ppo_loss(B, A, *[P(t) for t in args], float(clip), float(value_coef), float(entropy_coef),
                                 P(scratch), P(out), P(grad_mu), P(grad_std), P(grad_value), _stream(mu.device)))
        ctx.grads = (grad_mu, grad_std, grad_value)
        loss, stats = out[4], out[:4]
        ctx.mark_non_differentiable(stats)
        return loss, stats

    @staticmethod
    def backward(ctx, grad_loss, grad_stats):
        gm, gs, gv = ctx.grads
        return (gm * grad_loss, gs * grad_loss, gv * grad_loss) + (None,) * 10


def ppo_loss(policy, obs, critic_obs, actions, old_log_prob, old_mu, old_sigma, target_values, returns, advantages,
             cfg: PPOConfig):
    """Clipped surrogate + clipped value loss - entropy bonus (rsl-rl
    PPO.update); also the mean KL of the new policy to the old one."""
    if cfg.fused_loss and obs.is_cuda:
        mu = policy.mean(obs)
        value = policy.value(critic_obs)
        loss, stats = FusedPPOLoss.apply(mu, policy.std, value, actions, old_log_prob, old_mu, old_sigma,
                                         target_values, returns, advantages, cfg.clip, cfg.value_coef,
                                         cfg.entropy_coef)
        return loss, dict(surrogate=stats[0], value=stats[1], entropy=stats[2], kl=stats[3])
    dist_new = policy.distribution(obs)
    log_prob = dist_new.log_prob(actions).sum(-1)
    entropy = dist_new.entropy().sum(-1)
    mu, sigma = dist_new.mean, dist_new.stddev
    value = policy.value(critic_obs)
    kl = (torch.log(sigma / old_sigma + 1e-5)
          + (old_sigma.square() + (old_mu - mu).square()) / (2.0 * sigma.square()) - 0.5).sum(-1).mean()
    ratio = torch.exp(log_prob - old_log_prob)
    surrogate = torch.max(-advantages * ratio, -advantages * ratio.clamp(1.0 - cfg.clip, 1.0 + cfg.clip)).mean()
    clipped = target_values + (value - target_values).clamp(-cfg.clip, cfg.clip)
    value_loss = torch.max((value - returns).square(), (clipped - returns).square()).mean()
    loss = surrogate + cfg.value_coef * value_loss - cfg.entropy_coef * entropy.mean()
    return loss, dict(surrogate=surrogate.detach(), value=value_loss.detach(), entropy=entropy.mean().detach(),
                      kl=kl.detach())


class GradientAllReduce:
    """Averages gradients over the ranks of the default process group with one
    in-place all-reduce per bucket of about ``bucket_mb`` MB, issued from
    gradient hooks as soon as every parameter of the bucket has its gradient,
    so communication overlaps the rest of the backward pass."""

    def __init__(self, params, bucket_mb):
        self.world = dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
        self.params = [p for p in params if p.requires_grad]
        self.buckets, self.handles, self.pending = [], [], {}
        self.enabled = True   # off once a captured update averages the gradients itself
        if self.world == 1:
            return
        limit = max(1, int(bucket_mb * 1e6 / 4))
        bucket, size = [], 0
        for p in reversed(self.params):     # gradients arrive roughly in reverse order
            bucket.append(p)
            size += p.numel()
            if size >= limit:
                self.buckets.append(bucket)
                bucket, size = [], 0
        if bucket:
            self.buckets.append(bucket)
        self.flat = [torch.zeros(sum(p.numel() for p in b), device=b[0].device) for b in self.buckets]
        self.owner = {}
        for i, b in enumerate(self.buckets):
            for p in b:
                self.owner[p] = i
                p.register_post_accumulate_grad_hook(self._ready)

    def _ready(self, p):
        if not self.enabled:
            return
        i = self.owner[p]
        self.pending[i] = self.pending.get(i, 0) + 1
        if self.pending[i] == len(self.buckets[i]):
            flat, offset = self.flat[i], 0
            for q in self.buckets[i]:
                n = q.numel()
                flat[offset:offset + n].copy_(q.grad.reshape(-1))
                offset += n
            self.handles.append((i, dist.all_reduce(flat, async_op=True)))

    def finish(self):
        """Wait for the bucket all-reduces and write the averages back."""
        if self.world == 1 or not self.enabled:
            return
        if len(self.handles) != len(self.buckets):
            raise RuntimeError("a gradient bucket was not reduced (unused parameters?)")
        for i, handle in self.handles:
            handle.wait()
            flat, offset = self.flat[i], 0
            flat.div_(self.world)
            for q in self.buckets[i]:
                n = q.numel()
                q.grad.copy_(flat[offset:offset + n].view_as(q.grad))
                offset += n
        self.handles, self.pending = [], {}


def kl_schedule_host(lr: float, kl: float, desired: float) -> float:
    """rsl-rl's adaptive learning rate (rsl_rl/algorithms/ppo.py, the
    "adaptive" schedule): divide by 1.5 (not below 1e-5) when the KL exceeds
    twice the desired value, multiply by 1.5 (not above 1e-2) when it is
    positive and below half of it."""
    if kl > 2.0 * desired:
        return max(1e-5, lr / 1.5)
    if 0.0 < kl < desired / 2.0:
        return min(1e-2, lr * 1.5)
    return lr


def kl_schedule(lr: torch.Tensor, kl: torch.Tensor, desired: float) -> torch.Tensor:
    """kl_schedule_host on device tensors (float64 learning rate; the KL is
    compared in float64 like the host rule's Python floats)."""
    kl = kl.double()
    down = torch.clamp(lr / 1.5, min=1e-5)
    up = torch.clamp(lr * 1.5, max=1e-2)
    return torch.where(kl > 2.0 * desired, down, torch.where((kl > 0.0) & (kl < desired / 2.0), up, lr))


class PPO:
    """Rollout and update over an env with the rsl-rl VecEnv contract:
    ``get_observations()`` -> {"actor", "critic"} (or a tensor), ``step(actions)``
    -> (obs, reward, done, info) with ``info["time_outs"]``."""

    def __init__(self, env, cfg: PPOConfig | None = None, device=None, seed=0):
        self.cfg = cfg or PPOConfig()
        self.env = env
        self.device = torch.device(device or getattr(env, "device", "cuda"))
        torch.manual_seed(seed)
        obs = self._split(env.get_observations())
        self.obs, self.critic_obs = obs
        self.policy = ActorCritic(self.obs.shape[1], self.critic_obs.shape[1], env.num_actions, self.cfg).to(
            self.device)
        self.world = dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
        if self.world > 1:
            for p in self.policy.parameters():   # every rank starts from rank 0's weights
                dist.broadcast(p.data, 0)
        self.reducer = GradientAllReduce(self.policy.parameters(), self.cfg.bucket_mb)
        # On the GPU the learning rate lives on the device (fused Adam reads it
        # there) and the KL schedule updates it there, so an update never
        # waits for the host; on the CPU it is a Python float.
        if self.device.type == "cuda":
            self._lr64 = torch.tensor(self.cfg.learning_rate, dtype=torch.float64, device=self.device)
            self._lr = self._lr64.float()
            self.optimizer = torch.optim.Adam(self.policy.parameters(), lr=self._lr, fused=True, capturable=True)
        else:
            self._lr64 = self._lr = None
            self.optimizer = torch.optim.Adam(self.policy.parameters(), lr=self.cfg.learning_rate)
            self._host_lr = self.cfg.learning_rate
        self._graph = None
        self._updates, self._ugraphs, self._flat_grad = 0, None, None
        self.storage = Storage(self.cfg.steps_per_env, env.num_envs, self.obs.shape[1], self.critic_obs.shape[1],
                               env.num_actions, self.device)

    def _split(self, out):
        obs = out[0] if isinstance(out, tuple) else out
        if isinstance(obs, dict):
            return obs["actor"].to(self.device), obs["critic"].to(self.device)
        return obs.to(self.device), obs.to(self.device)

    def _act(self, obs, critic_obs):
        """One rollout step of the policy: sampled actions, their summed log
        probability, the distribution's mean and std, and the value."""
        d = self.policy.distribution(obs)
        # mean + std * N(0, 1) drawn in place: the same draw as sample(), whose
        # torch.normal(mean, std) checks std >= 0 on the host (no graph).
        actions = d.rsample()
        return actions, d.log_prob(actions).sum(-1), d.mean, d.stddev, self.policy.value(critic_obs)

    def _act_graphed(self, obs, critic_obs):
        """_act replayed from a CUDA graph: the policy's 30-odd small kernels
        are one launch, so a rollout step no longer waits on the host.  The
        graph reads the parameters in place, so it stays valid across
        optimizer steps; the samples come from the default CUDA generator."""
        if self._graph is None:
            self._graph_in = (obs.clone(), critic_obs.clone())
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                for _ in range(2):
                    self._act(*self._graph_in)
            torch.cuda.current_stream(self.device).wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                self._graph_out = self._act(*self._graph_in)
            self._graph = graph
        self._graph_in[0].copy_(obs)
        self._graph_in[1].copy_(critic_obs)
        self._graph.replay()
        return self._graph_out

    @torch.no_grad()
    def rollout(self):
        s, cfg = self.storage, self.cfg
        act = self._act_graphed if self.device.type == "cuda" and cfg.graph_rollout else self._act
        for t in range(cfg.steps_per_env):
            actions, log_prob, mu, sigma, values = act(self.obs, self.critic_obs)
            s.obs[t], s.critic_obs[t] = self.obs, self.critic_obs
            s.actions[t] = actions
            s.log_prob[t] = log_prob
            s.mu[t], s.sigma[t] = mu, sigma
            s.values[t] = values
            obs, reward, done, info = self.env.step(s.actions[t])
            reward = reward.to(self.device).float()
            if "time_outs" in info:
                reward = reward + cfg.gamma * s.values[t] * info["time_outs"].to(self.device).float()
            s.rewards[t] = reward
            s.dones[t] = done.to(self.device).float()
            self.obs, self.critic_obs = self._split(obs)
        last = self.policy.value(self.critic_obs)
        returns, advantages = gae(s.rewards, s.dones, s.values, last, cfg.gamma, cfg.lam)
        s.returns.copy_(returns)   # in place: a captured update reads these buffers
        s.advantages.copy_((advantages - advantages.mean()) / (advantages.std() + 1e-8))

    STATS = ("surrogate", "value", "entropy", "kl")

    def update(self, generator=None):
        """epochs x mini_batches PPO steps over the last rollout.  Every
        update after the first (which also creates the optimizer state) runs
        the minibatch step over a flat gradient buffer (_update_flat); on the
        GPU that step is replayed from CUDA graphs, so no step waits on the
        host.  The minibatch order is drawn eagerly either way."""
        if self.cfg.graph_update and self._updates > 0:
            return self._update_flat(generator)
        self._updates += 1
        s, cfg = self.storage, self.cfg
        n = s.T * s.E
        flat = lambda x: x.reshape(n, *x.shape[2:])
        data = [flat(x) for x in (s.obs, s.critic_obs, s.actions, s.log_prob, s.mu, s.sigma, s.values, s.returns,
                                  s.advantages)]
        size = n // cfg.mini_batches
        stats = []
        for _ in range(cfg.epochs):
            order = torch.randperm(n, device=self.device, generator=generator)
            for b in range(cfg.mini_batches):
                idx = order[b * size:(b + 1) * size]
                loss, info = ppo_loss(self.policy, *[x[idx] for x in data], cfg)
                self._adapt(info["kl"])
                self.optimizer.zero_grad(set_to_none=False)
                loss.backward()
                self.reducer.finish()
                nn.utils.clip_grad_norm_(self.policy.parameters(), cfg.max_grad_norm)
                with warnings.catch_warnings():   # capturable Adam stepped outside a graph
                    warnings.simplefilter("ignore", UserWarning)
                    self.optimizer.step()
                stats.append(info)
        return {k: torch.stack([x[k] for x in stats]).mean().item() for k in stats[0]}

    def _step_loss(self):
        """Forward and backward of one minibatch (the rows self._idx of the
        rollout), the KL in the last slot of the flat gradient buffer."""
        data = [x.index_select(0, self._idx) for x in self._data]
        loss, info = ppo_loss(self.policy, *data, self.cfg)
        self.optimizer.zero_grad(set_to_none=False)
        loss.backward()
        self._flat_grad[-1:].copy_(info["kl"].reshape(1))
        self._stats.copy_(torch.stack([info[k] for k in self.STATS]))

    def _step_apply(self):
        """KL learning-rate schedule, gradient clipping and the Adam step."""
        if self.cfg.desired_kl is not None and self._lr64 is not None:
            self._lr64.copy_(kl_schedule(self._lr64, self._flat_grad[-1], self.cfg.desired_kl))
            self._lr.copy_(self._lr64)
        elif self.cfg.desired_kl is not None:
            self._host_lr = kl_schedule_host(self._host_lr, float(self._flat_grad[-1]), self.cfg.desired_kl)
            for group in self.optimizer.param_groups:
                group["lr"] = self._host_lr
        nn.utils.clip_grad_norm_(self.policy.parameters(), self.cfg.max_grad_norm)
        self.optimizer.step()

    def _prepare_flat(self):
        s, cfg = self.storage, self.cfg
        n = s.T * s.E
        self._data = [x.reshape(n, *x.shape[2:]) for x in (s.obs, s.critic_obs, s.actions, s.log_prob, s.mu,
                                                             s.sigma, s.values, s.returns, s.advantages)]
        self._idx = torch.zeros(n // cfg.mini_batches, dtype=torch.long, device=self.device)
        self._stats = torch.zeros(len(self.STATS), device=self.device)
        # The gradients become views of one flat buffer (plus a KL slot), so
        # with several ranks one all-reduce between the two graphs averages
        # the gradients and the KL together.
        params = [p for p in self.policy.parameters() if p.requires_grad]
        total = sum(p.numel() for p in params)
        self._flat_grad = torch.zeros(total + 1, device=self.device)
        offset = 0
        for p in params:
            view = self._flat_grad[offset:offset + p.numel()].view_as(p)
            view.copy_(p.grad if p.grad is not None else torch.zeros_like(p))
            p.grad = view
            offset += p.numel()
        self.reducer.enabled = False
        # One part per side of the gradient all-reduce.
        self._parts = [[self._step_loss, self._step_apply]] if self.world == 1 else [[self._step_loss],
                                                                                      [self._step_apply]]
        if self.device.type == "cuda":
            graphs = []
            for fns in self._parts:
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    for fn in fns:
                        fn()
                graphs.append(graph)
            self._ugraphs = graphs

    def _run_part(self, i):
        if self._ugraphs is not None:
            self._ugraphs[i].replay()
        else:
            for fn in self._parts[i]:
                fn()

    def _update_flat(self, generator):
        s, cfg = self.storage, self.cfg
        if self._flat_grad is None:
            self._prepare_flat()
        n = s.T * s.E
        size = n // cfg.mini_batches
        stats = torch.empty(cfg.epochs * cfg.mini_batches, len(self.STATS), device=self.device)
        k = 0
        for _ in range(cfg.epochs):
            order = torch.randperm(n, device=self.device, generator=generator)
            for b in range(cfg.mini_batches):
                self._idx.copy_(order[b * size:(b + 1) * size])
                self._run_part(0)
                if self.world > 1:
                    dist.all_reduce(self._flat_grad)
                    self._flat_grad.div_(self.world)
                    self._run_part(1)
                stats[k].copy_(self._stats)
                k += 1
        means = stats.mean(0).tolist()
        return dict(zip(self.STATS, means))

    @property
    def learning_rate(self) -> float:
        return float(self._lr64) if self._lr64 is not None else self._host_lr

    def _adapt(self, kl):
        """rsl-rl's adaptive schedule: lr / 1.5 above 2 x desired KL, x 1.5
        below half of it (the KL averaged over ranks)."""
        if self.cfg.desired_kl is None:
            return
        if self.world > 1:
            kl = kl.clone()
            dist.all_reduce(kl)
            kl /= self.world
        if self._lr64 is not None:
            self._lr64.copy_(kl_schedule(self._lr64, kl, self.cfg.desired_kl))
            self._lr.copy_(self._lr64)
            return
        self._host_lr = kl_schedule_host(self._host_lr, float(kl), self.cfg.desired_kl)
        for group in self.optimizer.param_groups:
            group["lr"] = self._host_lr

    def learn(self, iterations):
        history = []
        for _ in range(iterations):
            self.rollout()
            history.append(self.update())
        return history
