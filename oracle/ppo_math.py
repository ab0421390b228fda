"""Restatement of the PPO algorithm in numpy -- TEST INFRASTRUCTURE ONLY (the
checker of duck_gym_b200/ppo.py).

The reference trains with rsl-rl's PPO (third-party package ``rsl_rl``,
version 5 per scripts/train_bam_native.py:1, not installed here).  Its
published algorithm, restated from the formulas, in float64:

* GAE: delta_t = r_t + gamma (1 - d_t) V_{t+1} - V_t,
  A_t = delta_t + gamma lambda (1 - d_t) A_{t+1}, returns R_t = A_t + V_t;
* surrogate: mean(max(-A ratio, -A clip(ratio, 1 - eps, 1 + eps)));
* clipped value loss: mean(max((V - R)^2, (V_old + clip(V - V_old) - R)^2));
* diagonal-Gaussian log-probabilities, entropies and KL divergence.
"""

import numpy as np


def gae(rewards, dones, values, last_values, gamma, lam):
    T = rewards.shape[0]
    returns = np.zeros_like(rewards)
    adv = np.zeros_like(last_values)
    for t in range(T - 1, -1, -1):
        nxt = last_values if t == T - 1 else values[t + 1]
        live = 1.0 - dones[t]
        delta = rewards[t] + live * gamma * nxt - values[t]
        adv = delta + live * gamma * lam * adv
        returns[t] = adv + values[t]
    return returns, returns - values


def normal_log_prob(x, mu, sigma):
    return (-((x - mu) ** 2) / (2 * sigma ** 2) - np.log(sigma) - 0.5 * np.log(2 * np.pi)).sum(-1)


def normal_entropy(sigma):
    return (0.5 + 0.5 * np.log(2 * np.pi) + np.log(sigma)).sum(-1)


def ppo_terms(mu, sigma, value, actions, old_log_prob, old_mu, old_sigma, target_values, returns, advantages, clip):
    log_prob = normal_log_prob(actions, mu, sigma)
    ratio = np.exp(log_prob - old_log_prob)
    surrogate = np.maximum(-advantages * ratio, -advantages * np.clip(ratio, 1 - clip, 1 + clip)).mean()
    clipped = target_values + np.clip(value - target_values, -clip, clip)
    value_loss = np.maximum((value - returns) ** 2, (clipped - returns) ** 2).mean()
    entropy = normal_entropy(sigma).mean()
    kl = (np.log(sigma / old_sigma + 1e-5) + (old_sigma ** 2 + (old_mu - mu) ** 2) / (2 * sigma ** 2) - 0.5).sum(-1).mean()
    return dict(surrogate=surrogate, value=value_loss, entropy=entropy, kl=kl)
