"""Reinforcement learning: grid-world environments (GridWorld, CliffWalking, FrozenLake), a vectorised
environment, replay buffers (uniform and prioritised), policy / value networks, and DQN (with double-DQN
targets), REINFORCE, A2C and PPO-clip agents.

Reference: crates/brain-rl. Environments (env/gridworld.rs:21-170, env/vector.rs), buffers
(buffer/mod.rs:25-100, buffer/prioritized.rs), DQN (dqn/mod.rs:31-140, dqn/double.rs), PPO clipped
objective (ppo/clipped.rs:17-45), A2C (a2c/mod.rs:20-90), categorical policies (policy/dist.rs),
discounted returns and GAE (utils.rs).

Objectives follow Mnih et al. 2015 (DQN), van Hasselt et al. 2016 (double DQN), Schulman et al. 2016
(GAE) and 2017 (PPO-clip). Networks use ``brain_b200.nn.Linear`` and run on any device.
"""
from __future__ import annotations

import math
import random
from collections import deque
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from ..nn.layers import Linear
from ..nn.module import Module


@dataclass
class Transition:
    state: torch.Tensor
    action: int
    reward: float
    next_state: torch.Tensor
    done: bool


class GridWorldEnv:
    """Agent starts at (0, 0) and must reach (w−1, h−1): reward −0.01 per step, +1 at the goal, episode
    capped at ``max_steps``. Actions 0..3 = up, right, down, left. Observation is a one-hot state."""

    ACTIONS = ((0, -1), (1, 0), (0, 1), (-1, 0))

    def __init__(self, width: int = 4, height: int = 4, max_steps: int = 100):
        self.w, self.h, self.max_steps = width, height, max_steps
        self.num_states, self.num_actions = width * height, 4
        self.reset()

    def state_index(self) -> int:
        return self.y * self.w + self.x

    def obs(self) -> torch.Tensor:
        o = torch.zeros(self.num_states)
        o[self.state_index()] = 1
        return o

    def reset(self) -> torch.Tensor:
        self.x = self.y = self.t = 0
        return self.obs()

    def _move(self, a: int):
        dx, dy = self.ACTIONS[a]
        self.x = min(max(self.x + dx, 0), self.w - 1)
        self.y = min(max(self.y + dy, 0), self.h - 1)

    def step(self, a: int):
        self._move(a)
        self.t += 1
        goal = self.x == self.w - 1 and self.y == self.h - 1
        done = goal or self.t >= self.max_steps
        return self.obs(), (1.0 if goal else -0.01), done, {}


class CliffWalkingEnv(GridWorldEnv):
    """4x12 grid; start bottom-left, goal bottom-right; the bottom row between them is a cliff (−100,
    back to start). −1 per step."""

    def __init__(self, max_steps: int = 200):
        super().__init__(12, 4, max_steps)

    def reset(self):
        self.x, self.y, self.t = 0, 3, 0
        return self.obs()

    def step(self, a):
        self._move(a)
        self.t += 1
        if self.y == 3 and 0 < self.x < 11:
            self.x, self.y = 0, 3
            return self.obs(), -100.0, self.t >= self.max_steps, {}
        goal = self.y == 3 and self.x == 11
        return self.obs(), -1.0, goal or self.t >= self.max_steps, {}


class FrozenLakeEnv(GridWorldEnv):
    """size x size lake with holes at a fixed seeded pattern (never start or goal); falling in ends the
    episode with 0 reward; reaching the goal gives 1. Deterministic moves (no slip)."""

    def __init__(self, size: int = 4, hole_fraction: float = 0.2, seed: int = 0, max_steps: int = 100):
        super().__init__(size, size, max_steps)
        rng = random.Random(seed)
        cells = [(x, y) for x in range(size) for y in range(size) if (x, y) not in ((0, 0), (size - 1, size - 1))]
        self.holes = set(rng.sample(cells, int(hole_fraction * size * size)))
        # keep the goal reachable along the top row and right column
        self.holes -= {(x, 0) for x in range(size)} | {(size - 1, y) for y in range(size)}

    def step(self, a):
        self._move(a)
        self.t += 1
        if (self.x, self.y) in self.holes:
            return self.obs(), 0.0, True, {"hole": True}
        goal = self.x == self.w - 1 and self.y == self.h - 1
        return self.obs(), (1.0 if goal else 0.0), goal or self.t >= self.max_steps, {}


class VectorEnv:
    """N copies stepped together; finished copies reset automatically."""

    def __init__(self, make_env, n: int):
        self.envs = [make_env() for _ in range(n)]

    def reset(self):
        return torch.stack([e.reset() for e in self.envs])

    def step(self, actions):
        obs, rew, done = [], [], []
        for e, a in zip(self.envs, actions):
            o, r, d, _ = e.step(int(a))
            if d:
                o = e.reset()
            obs.append(o)
            rew.append(r)
            done.append(d)
        return torch.stack(obs), torch.tensor(rew), torch.tensor(done)


class ReplayBuffer:
    def __init__(self, capacity: int, seed: int = 0):
        self.buf = deque(maxlen=capacity)
        self.rng = random.Random(seed)

    def __len__(self):
        return len(self.buf)

    def is_empty(self):
        return not self.buf

    def push(self, tr: Transition):
        self.buf.append(tr)

    def sample_batch(self, batch_size: int):
        if len(self.buf) < batch_size:
            raise ValueError(f"buffer holds {len(self.buf)} transitions, {batch_size} requested")
        return self.rng.sample(list(self.buf), batch_size)

    def stats(self) -> dict:
        r = [t.reward for t in self.buf]
        return {"len": len(r), "mean_reward": sum(r) / max(1, len(r))}


class PrioritizedReplayBuffer(ReplayBuffer):
    """Proportional prioritisation p_i^α with importance weights (N p_i)^−β / max (Schaul et al. 2016)."""

    def __init__(self, capacity: int, alpha: float = 0.6, beta: float = 0.4, seed: int = 0):
        super().__init__(capacity, seed)
        self.prio = deque(maxlen=capacity)
        self.alpha, self.beta = alpha, beta
        self.gen = torch.Generator().manual_seed(seed)

    def push(self, tr):
        super().push(tr)
        self.prio.append(max(self.prio, default=1.0))

    def sample_batch(self, batch_size):
        p = torch.tensor(list(self.prio), dtype=torch.float64) ** self.alpha
        p = p / p.sum()
        idx = torch.multinomial(p, batch_size, replacement=True, generator=self.gen)
        w = (len(p) * p[idx]) ** (-self.beta)
        self.last_idx = idx.tolist()
        return [self.buf[i] for i in self.last_idx], (w / w.max()).float()

    def update_priorities(self, td_errors):
        for i, e in zip(self.last_idx, td_errors):
            self.prio[i] = abs(float(e)) + 1e-6


class MlpNet(Module):
    def __init__(self, in_dim, out_dim, hidden=64, device=None, dtype=None):
        super().__init__()
        self.l1 = Linear(in_dim, hidden, True, device, dtype)
        self.l2 = Linear(hidden, hidden, True, device, dtype)
        self.l3 = Linear(hidden, out_dim, True, device, dtype)

    def forward(self, x):
        return self.l3(torch.relu(self.l2(torch.relu(self.l1(x)))))


def discounted_returns(rewards, dones, gamma: float) -> torch.Tensor:
    out, g = [], 0.0
    for r, d in zip(reversed(list(rewards)), reversed(list(dones))):
        g = float(r) + gamma * g * (0.0 if d else 1.0)
        out.append(g)
    return torch.tensor(out[::-1])


def gae(rewards, values, dones, gamma: float = 0.99, lam: float = 0.95, last_value: float = 0.0):
    """Generalised advantage estimates and returns (advantages + values)."""
    adv, a = [], 0.0
    values = list(map(float, values)) + [float(last_value)]
    for t in range(len(rewards) - 1, -1, -1):
        nonterm = 0.0 if dones[t] else 1.0
        delta = float(rewards[t]) + gamma * values[t + 1] * nonterm - values[t]
        a = delta + gamma * lam * nonterm * a
        adv.append(a)
    adv = torch.tensor(adv[::-1])
    return adv, adv + torch.tensor(values[:-1])


@dataclass
class DqnConfig:
    gamma: float = 0.99
    lr: float = 1e-3
    batch_size: int = 32
    buffer_capacity: int = 10000
    epsilon_start: float = 1.0
    epsilon_end: float = 0.05
    epsilon_decay_steps: int = 1000
    target_update: int = 100
    double: bool = True
    hidden: int = 64


class DqnAgent:
    def __init__(self, input_dim: int, num_actions: int, config: DqnConfig | None = None, seed: int = 0):
        self.c = config or DqnConfig()
        torch.manual_seed(seed)
        self.q = MlpNet(input_dim, num_actions, self.c.hidden)
        self.target = MlpNet(input_dim, num_actions, self.c.hidden)
        self.target.load_state_dict(self.q.state_dict())
        self.opt = torch.optim.Adam(self.q.parameters(), lr=self.c.lr)
        self.buffer = ReplayBuffer(self.c.buffer_capacity, seed)
        self.num_actions, self.steps = num_actions, 0
        self.rng = random.Random(seed)

    def epsilon(self) -> float:
        f = min(1.0, self.steps / max(1, self.c.epsilon_decay_steps))
        return self.c.epsilon_start + f * (self.c.epsilon_end - self.c.epsilon_start)

    def act(self, state, greedy: bool = False) -> int:
        if not greedy and self.rng.random() < self.epsilon():
            return self.rng.randrange(self.num_actions)
        with torch.no_grad():
            return int(self.q(state[None]).argmax())

    def step(self, tr: Transition) -> float:
        self.buffer.push(tr)
        self.steps += 1
        if len(self.buffer) < self.c.batch_size:
            return 0.0
        batch = self.buffer.sample_batch(self.c.batch_size)
        s = torch.stack([t.state for t in batch])
        a = torch.tensor([t.action for t in batch])
        r = torch.tensor([t.reward for t in batch])
        s2 = torch.stack([t.next_state for t in batch])
        d = torch.tensor([float(t.done) for t in batch])
        with torch.no_grad():
            if self.c.double:  # online net picks, target net evaluates
                a2 = self.q(s2).argmax(1, keepdim=True)
                q2 = self.target(s2).gather(1, a2).squeeze(1)
            else:
                q2 = self.target(s2).max(1).values
            y = r + self.c.gamma * (1 - d) * q2
        q = self.q(s).gather(1, a[:, None]).squeeze(1)
        loss = F.smooth_l1_loss(q, y)
        self.opt.zero_grad()
        loss.backward()
        self.opt.step()
        if self.steps % self.c.target_update == 0:
            self.target.load_state_dict(self.q.state_dict())
        return float(loss)


class PpoClippedObjective:
    def __init__(self, clip_epsilon: float = 0.2):
        self.eps = clip_epsilon

    def compute_policy_loss(self, ratio, advantage):
        ratio, advantage = torch.as_tensor(ratio), torch.as_tensor(advantage)
        return -torch.min(ratio * advantage, ratio.clamp(1 - self.eps, 1 + self.eps) * advantage).mean()

    def compute_value_loss(self, v_pred, v_old, v_target):
        v_pred, v_old, v_target = map(torch.as_tensor, (v_pred, v_old, v_target))
        clipped = v_old + (v_pred - v_old).clamp(-self.eps, self.eps)
        return 0.5 * torch.max((v_pred - v_target) ** 2, (clipped - v_target) ** 2).mean()


class ActorCritic(Module):
    def __init__(self, in_dim, num_actions, hidden=64, device=None, dtype=None):
        super().__init__()
        self.body = MlpNet(in_dim, hidden, hidden, device, dtype)
        self.pi = Linear(hidden, num_actions, True, device, dtype)
        self.v = Linear(hidden, 1, True, device, dtype)

    def forward(self, x):
        h = torch.relu(self.body(x))
        return self.pi(h), self.v(h).squeeze(-1)

    def dist(self, x):
        logits, v = self(x)
        return torch.distributions.Categorical(logits=logits), v


def rollout(env, policy: ActorCritic, steps: int, generator=None):
    """Collects ``steps`` transitions; returns states, actions, rewards, dones, log-probs, values."""
    S, A, R, D, LP, V = [], [], [], [], [], []
    s = env.reset()
    for _ in range(steps):
        with torch.no_grad():
            dist, v = policy.dist(s[None])
            a = int(dist.sample()[0])
            lp = float(dist.log_prob(torch.tensor([a]))[0])
        s2, r, d, _ = env.step(a)
        S.append(s), A.append(a), R.append(r), D.append(d), LP.append(lp), V.append(float(v[0]))
        s = env.reset() if d else s2
    return torch.stack(S), torch.tensor(A), R, D, torch.tensor(LP), V


@dataclass
class A2cConfig:
    gamma: float = 0.99
    lr: float = 3e-3
    value_coef: float = 0.5
    entropy_coef: float = 0.01
    rollout: int = 32
    hidden: int = 64


class A2cAgent:
    def __init__(self, input_dim, num_actions, config: A2cConfig | None = None, seed: int = 0):
        self.c = config or A2cConfig()
        torch.manual_seed(seed)
        self.net = ActorCritic(input_dim, num_actions, self.c.hidden)
        self.opt = torch.optim.Adam(self.net.parameters(), lr=self.c.lr)

    def act(self, state) -> int:
        with torch.no_grad():
            return int(self.net(state[None])[0].argmax())

    def update(self, env) -> float:
        S, A, R, D, _, V = rollout(env, self.net, self.c.rollout)
        ret = discounted_returns(R, D, self.c.gamma)
        dist, v = self.net.dist(S)
        adv = ret - v.detach()
        loss = (-(dist.log_prob(A) * adv).mean() + self.c.value_coef * F.mse_loss(v, ret) -
                self.c.entropy_coef * dist.entropy().mean())
        self.opt.zero_grad()
        loss.backward()
        self.opt.step()
        return float(loss)


@dataclass
class PpoConfig:
    gamma: float = 0.99
    lam: float = 0.95
    clip: float = 0.2
    lr: float = 3e-3
    epochs: int = 4
    rollout: int = 128
    value_coef: float = 0.5
    entropy_coef: float = 0.01
    hidden: int = 64


class PpoAgent:
    def __init__(self, input_dim, num_actions, config: PpoConfig | None = None, seed: int = 0):
        self.c = config or PpoConfig()
        torch.manual_seed(seed)
        self.net = ActorCritic(input_dim, num_actions, self.c.hidden)
        self.opt = torch.optim.Adam(self.net.parameters(), lr=self.c.lr)
        self.obj = PpoClippedObjective(self.c.clip)

    def act(self, state) -> int:
        with torch.no_grad():
            return int(self.net(state[None])[0].argmax())

    def update(self, env) -> float:
        S, A, R, D, LP, V = rollout(env, self.net, self.c.rollout)
        adv, ret = gae(R, V, D, self.c.gamma, self.c.lam)
        adv = (adv - adv.mean()) / (adv.std() + 1e-8)
        V = torch.tensor(V)
        last = 0.0
        for _ in range(self.c.epochs):
            dist, v = self.net.dist(S)
            ratio = torch.exp(dist.log_prob(A) - LP)
            loss = (self.obj.compute_policy_loss(ratio, adv) + self.c.value_coef * self.obj.compute_value_loss(v, V, ret)
                    - self.c.entropy_coef * dist.entropy().mean())
            self.opt.zero_grad()
            loss.backward()
            self.opt.step()
            last = float(loss)
        return last


def evaluate(env, act_fn, episodes: int = 5) -> float:
    tot = 0.0
    for _ in range(episodes):
        s, done = env.reset(), False
        while not done:
            s, r, done, _ = env.step(act_fn(s))
            tot += r
    return tot / episodes


class DuelingQNet(Module):
    """Q(s, a) = V(s) + A(s, a) − mean_a A(s, a) (Wang et al. 2016; reference dqn/dueling.rs)."""

    def __init__(self, in_dim, num_actions, hidden=64, device=None, dtype=None):
        super().__init__()
        self.body = MlpNet(in_dim, hidden, hidden, device, dtype)
        self.v = Linear(hidden, 1, True, device, dtype)
        self.a = Linear(hidden, num_actions, True, device, dtype)

    def forward(self, x):
        h = torch.relu(self.body(x))
        adv = self.a(h)
        return self.v(h) + adv - adv.mean(-1, keepdim=True)


# --------------------------------------------------------------------------- soft actor-critic
@dataclass
class SacConfig:
    """crates/brain-rl/src/sac/mod.rs:SacConfig (same fields and defaults)."""
    gamma: float = 0.99
    tau: float = 0.005
    alpha: float = 0.2
    auto_entropy_tuning: bool = True
    target_entropy: float = -1.0
    lr: float = 3e-4
    hidden: int = 64


class SacAgent:
    """Soft actor-critic for continuous actions (Haarnoja et al. 2018): a tanh-squashed Gaussian policy,
    twin Q critics with Polyak-averaged targets, and a learned temperature alpha (``log_alpha``) driven
    towards ``target_entropy`` when ``auto_entropy_tuning``. The reference's ``SacAgent`` holds the
    configuration and ``alpha()``; the update here is the full algorithm."""

    def __init__(self, state_dim: int, action_dim: int, config: SacConfig | None = None, device=None, seed: int = 0):
        self.config = c = config or SacConfig()
        self.state_dim, self.action_dim = state_dim, action_dim
        torch.manual_seed(seed)
        self.actor = MlpNet(state_dim, 2 * action_dim, c.hidden, device)
        self.q1 = MlpNet(state_dim + action_dim, 1, c.hidden, device)
        self.q2 = MlpNet(state_dim + action_dim, 1, c.hidden, device)
        self.q1_t = MlpNet(state_dim + action_dim, 1, c.hidden, device)
        self.q2_t = MlpNet(state_dim + action_dim, 1, c.hidden, device)
        self.q1_t.load_state_dict(self.q1.state_dict())
        self.q2_t.load_state_dict(self.q2.state_dict())
        self.log_alpha = torch.tensor(math.log(c.alpha), device=device, requires_grad=True)
        self.opt_actor = torch.optim.Adam(self.actor.parameters(), lr=c.lr)
        self.opt_q = torch.optim.Adam(list(self.q1.parameters()) + list(self.q2.parameters()), lr=c.lr)
        self.opt_alpha = torch.optim.Adam([self.log_alpha], lr=c.lr)

    def alpha(self) -> float:
        return float(self.log_alpha.exp())

    def _policy(self, s):
        mu, log_std = self.actor(s).chunk(2, -1)
        log_std = log_std.clamp(-20, 2)
        std = log_std.exp()
        u = mu + std * torch.randn_like(mu)
        a = torch.tanh(u)
        # log-density of the squashed sample: Gaussian log-prob minus log|d tanh / du|
        logp = (-0.5 * ((u - mu) / std) ** 2 - log_std - 0.5 * math.log(2 * math.pi)).sum(-1)
        logp = logp - torch.log(1 - a.pow(2) + 1e-6).sum(-1)
        return a, logp, torch.tanh(mu)

    @torch.no_grad()
    def act(self, state, deterministic: bool = False) -> torch.Tensor:
        a, _, mean = self._policy(torch.as_tensor(state, dtype=torch.float32)[None])
        return (mean if deterministic else a)[0]

    def update(self, s, a, r, s2, done) -> dict:
        """One gradient step on a batch (tensors [B, ...]); returns the losses and alpha."""
        c = self.config
        r, done = r.reshape(-1).float(), done.reshape(-1).float()
        with torch.no_grad():
            a2, logp2, _ = self._policy(s2)
            x2 = torch.cat([s2, a2], -1)
            q_t = torch.minimum(self.q1_t(x2), self.q2_t(x2)).reshape(-1) - self.alpha() * logp2
            y = r + c.gamma * (1 - done) * q_t
        x = torch.cat([s, a], -1)
        q_loss = ((self.q1(x).reshape(-1) - y) ** 2).mean() + ((self.q2(x).reshape(-1) - y) ** 2).mean()
        self.opt_q.zero_grad()
        q_loss.backward()
        self.opt_q.step()
        an, logp, _ = self._policy(s)
        xn = torch.cat([s, an], -1)
        actor_loss = (self.alpha() * logp - torch.minimum(self.q1(xn), self.q2(xn)).reshape(-1)).mean()
        self.opt_actor.zero_grad()
        actor_loss.backward()
        self.opt_actor.step()
        alpha_loss = torch.zeros(())
        if c.auto_entropy_tuning:
            alpha_loss = -(self.log_alpha * (logp.detach() + c.target_entropy)).mean()
            self.opt_alpha.zero_grad()
            alpha_loss.backward()
            self.opt_alpha.step()
        with torch.no_grad():
            for net, tgt in ((self.q1, self.q1_t), (self.q2, self.q2_t)):
                for p, pt in zip(net.parameters(), tgt.parameters()):
                    pt.mul_(1 - c.tau).add_(p, alpha=c.tau)
        return {"q_loss": float(q_loss), "actor_loss": float(actor_loss), "alpha_loss": float(alpha_loss),
                "alpha": self.alpha()}


# --------------------------------------------------------------------------- world model and curiosity
class WorldModel(Module):
    """Predicts the next state and the reward from (state, action) (crates/brain-rl/src/world_model.rs):
    h = ReLU(W_e [s, a] + b_e), s' = W_s h + b_s + s (residual), r = w_r . h + b_r, with the reference's
    deterministic initial weights (sin(0.1337 i), cos(0.7331 i), sin(0.4242 i) times sqrt(2 / in_dim)).
    Batched and differentiable, so it trains with ``loss`` (state MSE + 0.5 reward MSE)."""

    def __init__(self, state_dim: int, action_dim: int, hidden_dim: int, device=None):
        super().__init__()
        self.state_dim, self.action_dim, self.hidden_dim = state_dim, action_dim, hidden_dim
        in_dim = state_dim + action_dim
        scale = math.sqrt(2.0 / in_dim)
        i_e = torch.arange(hidden_dim * in_dim, dtype=torch.float64)
        i_s = torch.arange(state_dim * hidden_dim, dtype=torch.float64)
        i_r = torch.arange(hidden_dim, dtype=torch.float64)
        f = dict(device=device, dtype=torch.float32)
        self.w_embed = torch.nn.Parameter((torch.sin(i_e * 0.1337) * scale).view(hidden_dim, in_dim).to(**f))
        self.b_embed = torch.nn.Parameter(torch.zeros(hidden_dim, **f))
        self.w_state = torch.nn.Parameter((torch.cos(i_s * 0.7331) * scale).view(state_dim, hidden_dim).to(**f))
        self.b_state = torch.nn.Parameter(torch.zeros(state_dim, **f))
        self.w_reward = torch.nn.Parameter((torch.sin(i_r * 0.4242) * scale).view(1, hidden_dim).to(**f))
        self.b_reward = torch.nn.Parameter(torch.zeros(1, **f))

    def predict(self, state, action):
        """(next state [.., state_dim], reward [..]) for state [.., state_dim], action [.., action_dim]."""
        state, action = torch.as_tensor(state, dtype=torch.float32), torch.as_tensor(action, dtype=torch.float32)
        if state.shape[-1] != self.state_dim or action.shape[-1] != self.action_dim:
            raise ValueError(f"world model expects state [.., {self.state_dim}] and action [.., {self.action_dim}]")
        h = torch.relu(torch.cat([state, action], -1) @ self.w_embed.t() + self.b_embed)
        return h @ self.w_state.t() + self.b_state + state, (h @ self.w_reward.t() + self.b_reward).squeeze(-1)

    def loss(self, state, action, target_next_state, target_reward):
        s_pred, r_pred = self.predict(state, action)
        target_next_state = torch.as_tensor(target_next_state, dtype=torch.float32)
        target_reward = torch.as_tensor(target_reward, dtype=torch.float32)
        return ((s_pred - target_next_state) ** 2).mean(-1).mean() + 0.5 * ((r_pred - target_reward) ** 2).mean()


class IntrinsicCuriosityModule(Module):
    """Curiosity reward from a forward model's error in a learned feature space (Pathak et al. 2017;
    crates/brain-rl/src/curiosity.rs): phi(s) = LeakyReLU_0.01(W_enc s + b), phi_pred = W_f [phi(s), a] + b,
    reward = eta / 2 * ||phi_pred - phi(s')||^2, with the reference's initial weights (sin(0.177 i),
    cos(0.288 i) times sqrt(2 / state_dim)). ``inverse_head`` adds the inverse-dynamics model (predict a
    from phi(s), phi(s')) whose loss trains the encoder, as in the published method."""

    def __init__(self, state_dim: int, action_dim: int, feature_dim: int, eta: float = 0.1, device=None):
        super().__init__()
        self.state_dim, self.action_dim, self.feature_dim, self.eta = state_dim, action_dim, feature_dim, eta
        scale = math.sqrt(2.0 / state_dim)
        in_fwd = feature_dim + action_dim
        f = dict(device=device, dtype=torch.float32)
        i_e = torch.arange(feature_dim * state_dim, dtype=torch.float64)
        i_f = torch.arange(feature_dim * in_fwd, dtype=torch.float64)
        self.w_enc = torch.nn.Parameter((torch.sin(i_e * 0.177) * scale).view(feature_dim, state_dim).to(**f))
        self.b_enc = torch.nn.Parameter(torch.zeros(feature_dim, **f))
        self.w_forward = torch.nn.Parameter((torch.cos(i_f * 0.288) * scale).view(feature_dim, in_fwd).to(**f))
        self.b_forward = torch.nn.Parameter(torch.zeros(feature_dim, **f))
        self.inverse_head = Linear(2 * feature_dim, action_dim, True, device)

    def encode_state(self, state):
        state = torch.as_tensor(state, dtype=torch.float32)
        if state.shape[-1] != self.state_dim:
            raise ValueError(f"curiosity module expects states [.., {self.state_dim}]")
        return torch.nn.functional.leaky_relu(state @ self.w_enc.t() + self.b_enc, 0.01)

    def forward_error(self, state, action, next_state):
        phi = self.encode_state(state)
        action = torch.as_tensor(action, dtype=torch.float32)
        if action.shape[-1] != self.action_dim:
            raise ValueError(f"curiosity module expects actions [.., {self.action_dim}]")
        pred = torch.cat([phi, action], -1) @ self.w_forward.t() + self.b_forward
        return ((pred - self.encode_state(next_state)) ** 2).sum(-1)

    def compute_intrinsic_reward(self, state, action, next_state):
        """eta / 2 * forward-model error (no gradient)."""
        with torch.no_grad():
            return 0.5 * self.eta * self.forward_error(state, action, next_state)

    def loss(self, state, action, next_state, beta: float = 0.2):
        """ICM training loss: (1 - beta) * inverse-dynamics MSE + beta * forward error."""
        phi, phi2 = self.encode_state(state), self.encode_state(next_state)
        inv = ((self.inverse_head(torch.cat([phi, phi2], -1)) - torch.as_tensor(action, dtype=torch.float32)) ** 2)
        return (1 - beta) * inv.mean() + beta * self.forward_error(state, action, next_state).mean()
