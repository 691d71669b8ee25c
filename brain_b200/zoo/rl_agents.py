"""Reinforcement-learning building blocks beyond the core agents: n-step and trajectory buffers,
categorical / diagonal-Gaussian distributions, tabular and linear Q-functions, a skill library,
double-DQN and Rainbow-style agents, a DQN trainer, evaluation reports, checkpoints, and a batched
trainer that drives a :mod:`brain_b200.zoo.rl_envs` environment of N instances on a GPU.

Reference: crates/brain-rl/src/buffer/sequence.rs (NStepBuffer, TrajectoryBuffer), policy/dist.rs
(CategoricalDist, DiagonalGaussianDist), policy/gaussian.rs (GaussianPolicy), value/qvalue.rs (QTable,
QNet), skill_library.rs (SkillLibrary), dqn/double.rs, dqn/rainbow.rs, trainer.rs (DqnTrainer),
eval.rs (evaluate_dqn, EvalReport), checkpoint.rs (RlCheckpoint), utils.rs (discount_returns,
moving_average).

Agents here learn from a whole minibatch per update as tensors (one forward/backward per batch on
the device) where the reference loops over transitions one at a time; the targets are the same
(double-DQN: the online net picks the next action, the target net values it). The reference's
``RainbowAgent`` only refreshes priorities and never changes its network; this one also takes the
importance-weighted gradient step its priorities are meant for.
"""
from __future__ import annotations

import copy
import math
import random
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from .rl import DqnConfig, DuelingQNet, MlpNet, PrioritizedReplayBuffer, ReplayBuffer, Transition


# ------------------------------------------------------------------------------------------ utils
def discount_returns(rewards, gamma: float) -> torch.Tensor:
    """G_t = r_t + gamma G_{t+1}, over the last dimension (batched)."""
    r = torch.as_tensor(rewards, dtype=torch.float64)
    out = torch.empty_like(r)
    g = torch.zeros(r.shape[:-1], dtype=torch.float64)
    for t in range(r.shape[-1] - 1, -1, -1):
        g = r[..., t] + gamma * g
        out[..., t] = g
    return out


def moving_average(returns, alpha: float) -> list[float]:
    """Exponential smoothing that starts at the first value."""
    out, avg = [], 0.0
    for i, r in enumerate(returns):
        avg = float(r) if i == 0 else (1.0 - alpha) * avg + alpha * float(r)
        out.append(avg)
    return out


# ------------------------------------------------------------------------------------------ buffers
class NStepBuffer:
    """Folds the last n transitions into one: discounted reward sum (stopping at the first done), the
    first state and action, the last next_state. Returns None until n transitions are held."""

    def __init__(self, n_steps: int, gamma: float):
        self.n_steps, self.gamma = max(int(n_steps), 1), gamma
        self.history: list[Transition] = []

    def push(self, t: Transition):
        self.history.append(t)
        if len(self.history) < self.n_steps:
            return None
        ret, g, done = 0.0, 1.0, False
        for s in self.history:
            ret += g * s.reward
            g *= self.gamma
            if s.done:
                done = True
                break
        first, last = self.history[0], self.history[-1]
        self.history.pop(0)
        return Transition(first.state, first.action, ret, last.next_state, done)


class TrajectoryBuffer:
    def __init__(self):
        self.trajectories: list[list[Transition]] = []

    def push_trajectory(self, traj):
        self.trajectories.append(list(traj))

    def __len__(self):
        return len(self.trajectories)

    def is_empty(self):
        return not self.trajectories


# ------------------------------------------------------------------------------------------ distributions
class CategoricalDist:
    """Softmax over logits (batched over leading dims); log_prob floors p at 1e-15, an out-of-range action
    gives -1e10; entropy skips p <= 1e-15."""

    def __init__(self, logits):
        self.logits = torch.as_tensor(logits, dtype=torch.float64)
        self.probs = torch.softmax(self.logits, dim=-1)

    @classmethod
    def from_logits(cls, logits):
        return cls(logits)

    def log_prob(self, action):
        a = torch.as_tensor(action, dtype=torch.long)
        k = self.probs.shape[-1]
        ok = (a >= 0) & (a < k)
        p = self.probs.gather(-1, a.clamp(0, k - 1).unsqueeze(-1)).squeeze(-1)
        out = torch.where(ok, p.clamp_min(1e-15).log(), torch.full_like(p, -1e10))
        return float(out) if out.dim() == 0 else out

    def entropy(self):
        p = self.probs
        h = -(torch.where(p > 1e-15, p * p.clamp_min(1e-300).log(), torch.zeros_like(p))).sum(-1)
        return float(h) if h.dim() == 0 else h

    def sample(self, generator=None):
        return torch.multinomial(self.probs.reshape(-1, self.probs.shape[-1]), 1, generator=generator).view(
            self.probs.shape[:-1])


class DiagonalGaussianDist:
    def __init__(self, mean, log_std):
        self.mean = torch.as_tensor(mean, dtype=torch.float64)
        self.log_std = torch.as_tensor(log_std, dtype=torch.float64)

    def log_prob(self, action):
        a = torch.as_tensor(action, dtype=torch.float64)
        var = torch.exp(2.0 * self.log_std)
        lp = (-0.5 * ((a - self.mean) ** 2 / var + torch.log(2.0 * math.pi * var))).sum(-1)
        return float(lp) if lp.dim() == 0 else lp

    def entropy(self):
        h = (0.5 + 0.5 * math.log(2.0 * math.pi) + self.log_std).sum(-1)
        return float(h) if h.dim() == 0 else h

    def sample(self, generator=None):
        eps = torch.randn(self.mean.shape, dtype=torch.float64, generator=generator)
        return self.mean + torch.exp(self.log_std) * eps


class GaussianPolicy:
    """A state-independent log-std vector (initialised to 0) around a given mean."""

    def __init__(self, action_dim: int):
        self.log_std = torch.zeros(action_dim, dtype=torch.float64)

    def distribution(self, mean) -> DiagonalGaussianDist:
        return DiagonalGaussianDist(mean, self.log_std.expand_as(torch.as_tensor(mean, dtype=torch.float64)))


# ------------------------------------------------------------------------------------------ values
class QTable:
    """Sparse tabular Q (missing entries read 0) with the one-step Q-learning update."""

    def __init__(self):
        self.table: dict[tuple[int, int], float] = {}

    def get(self, s: int, a: int) -> float:
        return self.table.get((s, a), 0.0)

    def set(self, s: int, a: int, v: float) -> None:
        self.table[(s, a)] = float(v)

    def max_q(self, s: int, num_actions: int) -> float:
        return max((self.get(s, a) for a in range(num_actions)), default=0.0) if num_actions else 0.0

    def update_q(self, s, a, r, s2, num_actions, gamma, alpha):
        cur = self.get(s, a)
        self.set(s, a, cur + alpha * (r + gamma * self.max_q(s2, num_actions) - cur))


class QNet(torch.nn.Module):
    """Linear Q-function q = W s + b (zero-initialised), evaluated for a batch of states at once."""

    def __init__(self, input_dim: int, num_actions: int, device=None, dtype=torch.float32):
        super().__init__()
        self.input_dim, self.num_actions = input_dim, num_actions
        self.weight = torch.nn.Parameter(torch.zeros(num_actions, input_dim, device=device, dtype=dtype))
        self.bias = torch.nn.Parameter(torch.zeros(num_actions, device=device, dtype=dtype))

    def forward(self, s):
        s = s.to(self.weight.dtype)[..., :self.input_dim]
        return F.linear(s, self.weight[:, :s.shape[-1]], self.bias)


# ------------------------------------------------------------------------------------------ skills
@dataclass
class SkillStep:
    state_embedding: list
    action: list
    reward: float
    description: str | None = None


@dataclass
class Skill:
    name: str
    goal_embedding: list
    steps: list = field(default_factory=list)
    cumulative_reward: float = 0.0
    success_count: int = 0


class SkillLibrary:
    """Named skills retrieved by cosine similarity of goal embeddings (the best strictly above a floor);
    inserting an existing name replaces its steps and reward and counts one more success."""

    def __init__(self):
        self.skills: list[Skill] = []

    def insert(self, skill: Skill) -> None:
        for s in self.skills:
            if s.name == skill.name:
                s.steps, s.cumulative_reward = skill.steps, skill.cumulative_reward
                s.success_count += 1
                return
        self.skills.append(skill)

    def search(self, query, min_similarity: float):
        if not self.skills:
            return None
        q = torch.as_tensor(query, dtype=torch.float64)
        best, best_sim = None, min_similarity
        for s in self.skills:
            g = torch.as_tensor(s.goal_embedding, dtype=torch.float64)
            if q.numel() == 0 or g.numel() != q.numel():
                sim = 0.0
            else:
                den = math.sqrt(float(q @ q) * float(g @ g))
                sim = 0.0 if den < 1e-12 else float(q @ g) / den
            if sim > best_sim:
                best, best_sim = s, sim
        return best

    def __len__(self):
        return len(self.skills)

    def is_empty(self):
        return not self.skills


# ------------------------------------------------------------------------------------------ agents
def _epsilon(c: DqnConfig, steps: int) -> float:
    f = min(1.0, steps / max(1, c.epsilon_decay_steps))
    return c.epsilon_start + f * (c.epsilon_end - c.epsilon_start)


def _stack(batch, device):
    s = torch.stack([t.state for t in batch]).float().to(device)
    a = torch.tensor([t.action for t in batch], device=device)
    r = torch.tensor([t.reward for t in batch], dtype=torch.float32, device=device)
    s2 = torch.stack([t.next_state for t in batch]).float().to(device)
    d = torch.tensor([float(t.done) for t in batch], device=device)
    return s, a, r, s2, d


class DoubleDqnAgent:
    """Double DQN on a linear QNet (the reference's network) or an MLP (hidden > 0): target
    r + gamma Q_target(s', argmax_a Q_online(s', a)), squared TD error, SGD at lr over the minibatch,
    target copied every ``target_update`` steps."""

    def __init__(self, input_dim: int, num_actions: int, config: DqnConfig | None = None, hidden: int = 0,
                 device=None, seed: int = 0):
        self.c = config or DqnConfig()
        torch.manual_seed(seed)
        self.device = torch.device(device or "cpu")
        self.q_online = (MlpNet(input_dim, num_actions, hidden) if hidden else QNet(input_dim, num_actions)).to(self.device)
        self.q_target = copy.deepcopy(self.q_online)
        self.opt = torch.optim.SGD(self.q_online.parameters(), lr=self.c.lr)
        self.buffer = ReplayBuffer(self.c.buffer_capacity, seed)
        self.num_actions, self.total_steps = num_actions, 0
        self.rng = random.Random(seed)

    def act(self, state, greedy: bool = False) -> int:
        if not greedy and self.rng.random() < _epsilon(self.c, self.total_steps):
            return self.rng.randrange(self.num_actions)
        with torch.no_grad():
            return int(self.q_online(state.float().to(self.device)[None]).argmax())

    def _targets(self, r, s2, d):
        with torch.no_grad():
            a2 = self.q_online(s2).argmax(1, keepdim=True)
            return r + self.c.gamma * (1.0 - d) * self.q_target(s2).gather(1, a2).squeeze(1)

    def step(self, tr: Transition) -> float:
        self.buffer.push(tr)
        self.total_steps += 1
        if len(self.buffer) < self.c.batch_size:
            return 0.0
        s, a, r, s2, d = _stack(self.buffer.sample_batch(self.c.batch_size), self.device)
        y = self._targets(r, s2, d)
        q = self.q_online(s).gather(1, a[:, None]).squeeze(1)
        loss = (y - q).pow(2).mean()
        self.opt.zero_grad()
        (0.5 * loss).backward()
        self.opt.step()
        if self.total_steps % self.c.target_update == 0:
            self.q_target.load_state_dict(self.q_online.state_dict())
        return float(loss.detach())


class RainbowAgent(DoubleDqnAgent):
    """Dueling network, prioritised replay (alpha 0.6, beta 0.4), n-step returns and double-DQN
    targets; the loss is the importance-weighted squared TD error and new priorities are
    max(|td|, 1e-5)^alpha."""

    def __init__(self, input_dim: int, num_actions: int, config: DqnConfig | None = None, n_steps: int = 3,
                 device=None, seed: int = 0):
        super().__init__(input_dim, num_actions, config, 0, device, seed)
        self.q_online = DuelingQNet(input_dim, num_actions, self.c.hidden).to(self.device)
        self.q_target = copy.deepcopy(self.q_online)
        self.opt = torch.optim.Adam(self.q_online.parameters(), lr=self.c.lr)
        self.per_buffer = PrioritizedReplayBuffer(self.c.buffer_capacity, 0.6, 0.4, seed)
        self.nstep = NStepBuffer(n_steps, self.c.gamma)
        self.n_steps = n_steps

    def step(self, tr: Transition) -> float:
        folded = self.nstep.push(tr)
        self.total_steps += 1
        if folded is not None:
            self.per_buffer.push(folded)
        if len(self.per_buffer) < self.c.batch_size:
            return 0.0
        batch, w = self.per_buffer.sample_batch(self.c.batch_size)
        s, a, r, s2, d = _stack(batch, self.device)
        with torch.no_grad():
            a2 = self.q_online(s2).argmax(1, keepdim=True)
            y = r + (self.c.gamma ** self.n_steps) * (1.0 - d) * self.q_target(s2).gather(1, a2).squeeze(1)
        q = self.q_online(s).gather(1, a[:, None]).squeeze(1)
        td = y - q
        loss = (w.to(self.device) * td.pow(2)).mean()
        self.opt.zero_grad()
        loss.backward()
        self.opt.step()
        self.per_buffer.update_priorities(td.detach().abs().clamp_min(1e-5).cpu())  # raised to alpha when sampled
        if self.total_steps % self.c.target_update == 0:
            self.q_target.load_state_dict(self.q_online.state_dict())
        return float(loss.detach())


# ------------------------------------------------------------------------------------------ training loops
@dataclass
class TrainerConfig:
    max_episodes: int = 100
    max_steps_per_episode: int = 500
    eval_freq: int = 10


class DqnTrainer:
    """Episode loop over a one-instance environment (``reset()`` / ``step(a) -> EnvStep``): act, step,
    store (done = done or truncated), learn; returns the per-episode rewards."""

    def __init__(self, agent, env, config: TrainerConfig | None = None):
        self.agent, self.env, self.config = agent, env, config or TrainerConfig()
        self.episode_rewards: list[float] = []

    def train(self) -> list[float]:
        for _ in range(self.config.max_episodes):
            s = self.env.reset()
            ep = 0.0
            for _ in range(self.config.max_steps_per_episode):
                a = self.agent.act(s)
                st = self.env.step(a)
                ep += st.reward
                self.agent.step(Transition(s, a, st.reward, st.observation, st.done or st.truncated))
                s = st.observation
                if st.done or st.truncated:
                    break
            self.episode_rewards.append(ep)
        return list(self.episode_rewards)


@dataclass
class EvalReport:
    num_episodes: int
    mean_return: float
    std_return: float
    min_return: float
    max_return: float


def evaluate_dqn(agent, env, num_episodes: int, max_steps: int = 1000) -> EvalReport:
    """Greedy returns over episodes (population standard deviation)."""
    if num_episodes <= 0:
        raise ValueError("num_episodes must be > 0")
    rets = []
    for _ in range(num_episodes):
        s, ep = env.reset(), 0.0
        for _ in range(max_steps):
            with torch.no_grad():
                a = int(agent.q_online(s.float().to(agent.device)[None]).argmax())
            st = env.step(a)
            ep += st.reward
            s = st.observation
            if st.done or st.truncated:
                break
        rets.append(ep)
    t = torch.tensor(rets, dtype=torch.float64)
    return EvalReport(num_episodes, float(t.mean()), float(t.std(unbiased=False)), float(t.min()), float(t.max()))


@dataclass
class RlCheckpoint:
    total_steps: int
    q_state: dict
    buffer_count: int

    @classmethod
    def save_dqn(cls, agent) -> "RlCheckpoint":
        return cls(agent.total_steps, {k: v.detach().cpu().clone() for k, v in agent.q_online.state_dict().items()},
                   len(agent.buffer))

    def load_dqn(self, agent) -> None:
        own = agent.q_online.state_dict()
        if set(own) != set(self.q_state) or any(own[k].shape != self.q_state[k].shape for k in own):
            raise ValueError("checkpoint weight shapes do not match the agent")
        agent.total_steps = self.total_steps
        agent.q_online.load_state_dict(self.q_state)
        agent.q_target.load_state_dict(self.q_state)


class BatchedDqnTrainer:
    """Double-DQN on N environment instances at once: every step acts for all N (epsilon-greedy on the
    device), stores N transitions in a device-resident circular replay, takes one minibatch gradient
    step, and resets finished instances in place. Nothing leaves the device inside the loop except the
    episode returns of instances that finished."""

    def __init__(self, env, hidden: int = 64, capacity: int = 100_000, batch_size: int = 256, lr: float = 1e-3,
                 gamma: float = 0.99, target_update: int = 200, eps_start: float = 1.0, eps_end: float = 0.05,
                 eps_decay_steps: int = 2000, seed: int = 0):
        from .rl_envs import _base
        base = _base(env)
        self.env, self.dev, self.n = env, base.device, env.n
        g = torch.Generator(device="cpu").manual_seed(seed)
        torch.manual_seed(seed)
        self.q = MlpNet(env.obs_dim, env.num_actions, hidden).to(self.dev)
        self.q_t = copy.deepcopy(self.q)
        self.opt = torch.optim.Adam(self.q.parameters(), lr=lr)
        self.cap, self.bs, self.gamma, self.tu = capacity, batch_size, gamma, target_update
        self.eps = (eps_start, eps_end, eps_decay_steps)
        d = env.obs_dim
        self.S = torch.zeros(capacity, d, device=self.dev)
        self.S2 = torch.zeros(capacity, d, device=self.dev)
        self.A = torch.zeros(capacity, dtype=torch.long, device=self.dev)
        self.R = torch.zeros(capacity, device=self.dev)
        self.D = torch.zeros(capacity, device=self.dev)
        self.ptr, self.size, self.steps = 0, 0, 0
        self.gen = torch.Generator(device=self.dev).manual_seed(seed)
        self.obs = env.reset().float()
        self.ret = torch.zeros(self.n, device=self.dev)
        self.finished: list[float] = []
        del g

    def _store(self, s, a, r, s2, d):
        idx = (self.ptr + torch.arange(self.n, device=self.dev)) % self.cap
        self.S[idx], self.A[idx], self.R[idx], self.S2[idx], self.D[idx] = s, a, r, s2, d
        self.ptr = (self.ptr + self.n) % self.cap
        self.size = min(self.size + self.n, self.cap)

    def step(self) -> float:
        e0, e1, k = self.eps
        eps = e0 + min(1.0, self.steps / max(1, k)) * (e1 - e0)
        with torch.no_grad():
            greedy = self.q(self.obs).argmax(1)
        rand = torch.randint(0, self.env.num_actions, (self.n,), device=self.dev, generator=self.gen)
        explore = torch.rand(self.n, device=self.dev, generator=self.gen) < eps
        a = torch.where(explore, rand, greedy)
        o2, r, done, trunc = self.env.step(a)
        o2, r = o2.float(), r.float()
        self._store(self.obs, a, r, o2, done.float())
        self.ret += r
        end = done | trunc
        if bool(end.any()):
            self.finished.extend(self.ret[end].tolist())
            self.ret[end] = 0.0
            o2 = torch.where(end[:, None], self.env.reset(end).float(), o2)
        self.obs = o2
        self.steps += 1
        if self.size < self.bs:
            return 0.0
        i = torch.randint(0, self.size, (self.bs,), device=self.dev, generator=self.gen)
        with torch.no_grad():
            a2 = self.q(self.S2[i]).argmax(1, keepdim=True)
            y = self.R[i] + self.gamma * (1.0 - self.D[i]) * self.q_t(self.S2[i]).gather(1, a2).squeeze(1)
        qv = self.q(self.S[i]).gather(1, self.A[i][:, None]).squeeze(1)
        loss = F.smooth_l1_loss(qv, y)
        self.opt.zero_grad()
        loss.backward()
        self.opt.step()
        if self.steps % self.tu == 0:
            self.q_t.load_state_dict(self.q.state_dict())
        return float(loss.detach())


# ------------------------------------------------------------------ the reference's names
# crates/brain-rl/src: env/{gym,atari_lite,mujoco_lite,wrappers,vector}.rs, dqn/dueling.rs,
# actor_critic/mod.rs (ActorCriticNet, compute_gae), policy/mod.rs (EpsilonSchedule, EpsilonGreedyPolicy),
# value/mod.rs (soft_update_target, VTable / update_td), buffer/prioritized.rs (SumTree), agents/mod.rs (make_agent).
from . import rl as _rl, rl_envs as _envs  # noqa: E402

CartPoleEnv = _envs.CartPole
MountainCarEnv = _envs.MountainCar
PendulumEnv = _envs.Pendulum
PongLiteEnv = _envs.PongLite
BreakoutLiteEnv = _envs.BreakoutLite
HalfCheetahLiteEnv = _envs.HalfCheetahLite
ReacherLiteEnv = _envs.ReacherLite
FrameStackWrapper = _envs.FrameStack
TimeLimitWrapper = _envs.TimeLimit
RewardScaleWrapper = _envs.RewardScale
DummyVecEnv = _rl.VectorEnv
ActorCriticNet = _rl.ActorCritic
compute_gae = _rl.gae


class EpsilonSchedule:
    """Linear decay from ``start`` to ``end`` over ``decay_steps``, then constant."""

    def __init__(self, start: float = 1.0, end: float = 0.05, decay_steps: int = 10000):
        self.start, self.end, self.decay = start, end, max(1, decay_steps)

    def get_epsilon(self, step: int) -> float:
        f = min(step / self.decay, 1.0)
        return self.start + f * (self.end - self.start)


class EpsilonGreedyPolicy:
    """Batched epsilon-greedy: random actions where a uniform draw is below epsilon, argmax elsewhere."""

    def __init__(self, schedule: EpsilonSchedule, num_actions: int, seed: int = 0):
        self.schedule, self.n = schedule, num_actions
        self.g = torch.Generator().manual_seed(seed)

    def select_action(self, q_values: torch.Tensor, step: int) -> torch.Tensor:
        eps = self.schedule.get_epsilon(step)
        greedy = q_values.argmax(-1)
        rnd = torch.randint(0, self.n, greedy.shape, generator=self.g).to(greedy.device)
        explore = (torch.rand(greedy.shape, generator=self.g) < eps).to(greedy.device)
        return torch.where(explore, rnd, greedy)


def soft_update_target(target: torch.nn.Module, source: torch.nn.Module, tau: float = 0.005) -> None:
    """theta_target <- tau theta + (1 - tau) theta_target (Polyak)."""
    with torch.no_grad():
        for t, s in zip(target.parameters(), source.parameters()):
            t.lerp_(s, tau)


class VTable:
    """Tabular state values with TD(0) updates."""

    def __init__(self, num_states: int, gamma: float = 0.99, lr: float = 0.1):
        self.v, self.gamma, self.lr = torch.zeros(num_states, dtype=torch.float64), gamma, lr

    def update_td(self, s: int, r: float, s_next: int, done: bool) -> float:
        target = r + (0.0 if done else self.gamma * float(self.v[s_next]))
        err = target - float(self.v[s])
        self.v[s] += self.lr * err
        return err


class SumTree:
    """Binary sum tree over ``capacity`` priorities: O(log n) update and prefix-sum sampling."""

    def __init__(self, capacity: int):
        self.cap = 1
        while self.cap < capacity:
            self.cap *= 2
        self.tree = [0.0] * (2 * self.cap)

    def update(self, idx: int, priority: float) -> None:
        i = idx + self.cap
        self.tree[i] = float(priority)
        i //= 2
        while i:
            self.tree[i] = self.tree[2 * i] + self.tree[2 * i + 1]
            i //= 2

    def total_priority(self) -> float:
        return self.tree[1]

    def get_leaf(self, value: float) -> tuple[int, float]:
        """(index, priority) of the leaf whose prefix-sum interval contains ``value``."""
        i = 1
        while i < self.cap:
            left = self.tree[2 * i]
            if value < left:
                i = 2 * i
            else:
                value -= left
                i = 2 * i + 1
        return i - self.cap, self.tree[i]


def make_agent(kind: str, obs_dim: int, num_actions: int, **kw):
    """Construct an agent by name: dqn, double_dqn, rainbow, a2c, ppo, sac."""
    table = {"dqn": (_rl.DqnAgent, _rl.DqnConfig), "double_dqn": (DoubleDqnAgent, _rl.DqnConfig),
             "rainbow": (RainbowAgent, _rl.DqnConfig), "a2c": (_rl.A2cAgent, _rl.A2cConfig),
             "ppo": (_rl.PpoAgent, _rl.PpoConfig), "sac": (_rl.SacAgent, _rl.SacConfig)}
    if kind not in table:
        raise ValueError(f"unknown agent {kind!r}")
    seed = kw.pop("seed", 0)
    cls, cfg = table[kind]
    return cls(obs_dim, num_actions, cfg(**kw), seed=seed)
