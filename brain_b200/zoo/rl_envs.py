"""Batched reinforcement-learning environments: N independent instances stepped by tensor operations.

Reference: crates/brain-rl/src/env/gym.rs (CartPole, MountainCar, Pendulum), env/atari_lite.rs
(PongLite, BreakoutLite), env/mujoco_lite.rs (HalfCheetahLite, ReacherLite), env/wrappers.rs
(frame stacking, time limit, reward scaling). The reference steps one instance per call on the host.
Here an environment holds a [N, ...] state tensor on any device (a GPU runs thousands of instances
in one step), ``step(actions [N])`` advances all of them with the reference's dynamics and returns
``(obs [N, d], reward [N], done [N], truncated [N])``, and ``reset(mask)`` restarts the selected
instances only, so an agent can auto-reset finished episodes without a host loop. Dynamics and
constants are the reference's (explicit Euler, the same thresholds, clamps, rewards and step caps);
``SingleEnv`` wraps any of them as the reference's one-instance ``reset() / step(action)`` API.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass
class EnvStep:
    observation: torch.Tensor
    reward: float
    done: bool
    truncated: bool


@dataclass
class Space:
    """Discrete(n) when ``n`` is set, else Continuous(shape, low, high)."""
    n: int | None = None
    shape: tuple = ()
    low: float = 0.0
    high: float = 0.0


class BatchedEnv:
    obs_dim = 0
    num_actions = 0
    max_steps = 0
    obs_low, obs_high = 0.0, 0.0

    def __init__(self, num_envs: int = 1, device=None, dtype=torch.float64):
        self.n, self.device, self.dtype = int(num_envs), torch.device(device or "cpu"), dtype
        self.t = torch.zeros(self.n, dtype=torch.long, device=self.device)
        self._init_state()
        self.reset()

    def _z(self, *shape):
        return torch.zeros(self.n, *shape, dtype=self.dtype, device=self.device)

    def _mask(self, mask):
        if mask is None:
            return torch.ones(self.n, dtype=torch.bool, device=self.device)
        return mask.to(self.device, torch.bool)

    def action_space(self) -> Space:
        return Space(n=self.num_actions)

    def observation_space(self) -> Space:
        return Space(shape=(self.obs_dim,), low=self.obs_low, high=self.obs_high)

    def _check(self, actions):
        a = torch.as_tensor(actions, device=self.device).long().reshape(self.n)
        if bool(((a < 0) | (a >= self.num_actions)).any()):
            raise ValueError(f"invalid action for a {self.num_actions}-action environment")
        return a

    def _finish(self, reward, done, cap):
        self.t += 1
        truncated = self.t >= cap
        return self.obs(), reward, done, truncated


class CartPole(BatchedEnv):
    """Pole on a cart: force +-10 N, Euler step tau 0.02 s, done when |x| > 2.4 or |theta| > 12 deg,
    reward 1 per step, truncated at 500 steps."""
    obs_dim, num_actions, max_steps, obs_low, obs_high = 4, 2, 500, -4.8, 4.8
    gravity, masscart, masspole, length, force_mag, tau = 9.8, 1.0, 0.1, 0.5, 10.0, 0.02
    theta_limit, x_limit = 12.0 * 2.0 * math.pi / 360.0, 2.4

    def _init_state(self):
        self.s = self._z(4)  # x, x_dot, theta, theta_dot

    def reset(self, mask=None):
        m = self._mask(mask)
        self.s[m] = 0.0
        self.t[m] = 0
        return self.obs()

    def obs(self):
        return self.s.clone()

    def step(self, actions):
        a = self._check(actions)
        x, xd, th, thd = self.s.unbind(1)
        force = torch.where(a == 1, self.force_mag, -self.force_mag).to(self.dtype)
        c, s = torch.cos(th), torch.sin(th)
        total = self.masscart + self.masspole
        pml = self.masspole * self.length
        temp = (force + pml * thd * thd * s) / total
        thacc = (self.gravity * s - c * temp) / (self.length * (4.0 / 3.0 - self.masspole * c * c / total))
        xacc = temp - pml * thacc * c / total
        self.s = torch.stack([x + self.tau * xd, xd + self.tau * xacc, th + self.tau * thd, thd + self.tau * thacc], 1)
        x, th = self.s[:, 0], self.s[:, 2]
        done = (x < -self.x_limit) | (x > self.x_limit) | (th < -self.theta_limit) | (th > self.theta_limit)
        return self._finish(torch.ones(self.n, dtype=self.dtype, device=self.device), done, self.max_steps)


class MountainCar(BatchedEnv):
    """Car in a valley: velocity += (a - 1) 0.001 - 0.0025 cos(3 x), clamped to +-0.07; position clamped to
    [-1.2, 0.6] (velocity zeroed at the left wall); done at x >= 0.5; reward -1; 200 steps."""
    obs_dim, num_actions, max_steps, obs_low, obs_high = 2, 3, 200, -1.2, 0.6

    def _init_state(self):
        self.s = self._z(2)

    def reset(self, mask=None):
        m = self._mask(mask)
        self.s[m] = torch.tensor([-0.5, 0.0], dtype=self.dtype, device=self.device)
        self.t[m] = 0
        return self.obs()

    def obs(self):
        return self.s.clone()

    def step(self, actions):
        a = self._check(actions).to(self.dtype)
        p, v = self.s.unbind(1)
        v = (v + (a - 1.0) * 0.001 + torch.cos(3.0 * p) * -0.0025).clamp(-0.07, 0.07)
        p = (p + v).clamp(-1.2, 0.6)
        v = torch.where((p <= -1.2) & (v < 0.0), torch.zeros_like(v), v)
        self.s = torch.stack([p, v], 1)
        return self._finish(torch.full((self.n,), -1.0, dtype=self.dtype, device=self.device), p >= 0.5, self.max_steps)


class Pendulum(BatchedEnv):
    """Torque u = (a - 1) 2 on a pendulum (g 10, m 1, l 1, dt 0.05): angular velocity clamped to +-8, cost
    th^2 + 0.1 thdot^2 + 0.001 u^2 on the unwrapped angle; never done, 200 steps. Obs (cos, sin, thdot)."""
    obs_dim, num_actions, max_steps, obs_low, obs_high = 3, 3, 200, -8.0, 8.0

    def _init_state(self):
        self.s = self._z(2)  # th, thdot

    def reset(self, mask=None):
        m = self._mask(mask)
        self.s[m] = 0.0
        self.t[m] = 0
        return self.obs()

    def obs(self):
        th, thd = self.s.unbind(1)
        return torch.stack([torch.cos(th), torch.sin(th), thd], 1)

    def step(self, actions):
        u = (self._check(actions).to(self.dtype) - 1.0) * 2.0
        th, thd = self.s.unbind(1)
        g, m, l, dt = 10.0, 1.0, 1.0, 0.05
        thd = (thd + (-3.0 * g / (2.0 * l) * torch.sin(th + math.pi) + 3.0 / (m * l * l) * u) * dt).clamp(-8.0, 8.0)
        th = th + thd * dt
        self.s = torch.stack([th, thd], 1)
        reward = -(th * th + 0.1 * thd * thd + 0.001 * u * u)
        return self._finish(reward, torch.zeros(self.n, dtype=torch.bool, device=self.device), self.max_steps)


class PongLite(BatchedEnv):
    """Paddle (0 stay, 1 up, 2 down by 0.05) against a ball bouncing off the walls: +1 for a return within
    0.15 of the paddle at x <= 0, -1 and done for a miss; 1000 steps. Obs (paddle_y, bx, by, vx, vy)."""
    obs_dim, num_actions, max_steps, obs_low, obs_high = 5, 3, 1000, 0.0, 1.0

    def _init_state(self):
        self.s = self._z(5)

    def reset(self, mask=None):
        m = self._mask(mask)
        self.s[m] = torch.tensor([0.5, 0.5, 0.5, 0.05, 0.03], dtype=self.dtype, device=self.device)
        self.t[m] = 0
        return self.obs()

    def obs(self):
        return self.s.clone()

    def step(self, actions):
        a = self._check(actions)
        py, bx, by, vx, vy = self.s.unbind(1)
        py = torch.where(a == 1, (py - 0.05).clamp_min(0.0), torch.where(a == 2, (py + 0.05).clamp_max(1.0), py))
        bx, by = bx + vx, by + vy
        vy = torch.where((by <= 0.0) | (by >= 1.0), -vy, vy)
        vx = torch.where(bx >= 1.0, -vx, vx)
        left = bx <= 0.0
        hit = left & ((by - py).abs() < 0.15)
        miss = left & ~hit
        vx = torch.where(hit, -vx, vx)
        reward = torch.where(hit, 1.0, torch.where(miss, -1.0, 0.0)).to(self.dtype)
        self.s = torch.stack([py, bx, by, vx, vy], 1)
        return self._finish(reward, miss, self.max_steps)


class BreakoutLite(BatchedEnv):
    """Paddle along the bottom returns a ball (+0.1) or misses it (-1, done); 500 steps. Obs (paddle_x, bx, by)."""
    obs_dim, num_actions, max_steps, obs_low, obs_high = 3, 3, 500, 0.0, 1.0

    def _init_state(self):
        self.s = self._z(5)  # paddle_x, bx, by, vx, vy
        self.bricks_left = torch.full((self.n,), 20, dtype=torch.long, device=self.device)

    def reset(self, mask=None):
        m = self._mask(mask)
        self.s[m] = torch.tensor([0.5, 0.5, 0.2, 0.04, 0.04], dtype=self.dtype, device=self.device)
        self.bricks_left[m] = 20
        self.t[m] = 0
        return self.obs()

    def obs(self):
        return self.s[:, :3].clone()

    def step(self, actions):
        a = self._check(actions)
        px, bx, by, vx, vy = self.s.unbind(1)
        px = torch.where(a == 1, (px - 0.05).clamp_min(0.0), torch.where(a == 2, (px + 0.05).clamp_max(1.0), px))
        bx, by = bx + vx, by + vy
        vx = torch.where((bx <= 0.0) | (bx >= 1.0), -vx, vx)
        vy = torch.where(by >= 1.0, -vy, vy)
        bottom = by <= 0.0
        hit = bottom & ((bx - px).abs() < 0.15)
        miss = bottom & ~hit
        vy = torch.where(hit, -vy, vy)
        reward = torch.where(hit, 0.1, torch.where(miss, -1.0, 0.0)).to(self.dtype)
        self.s = torch.stack([px, bx, by, vx, vy], 1)
        return self._finish(reward, miss, self.max_steps)


class HalfCheetahLite(BatchedEnv):
    """Forward-running body: torque (a - 1) 0.5 changes velocity by torque 0.1 (clamped to [-2, 5]),
    reward velocity - 0.1 torque^2; never done, 1000 steps. Obs (x, v, six joint angles)."""
    obs_dim, num_actions, max_steps, obs_low, obs_high = 8, 3, 1000, -10.0, 10.0

    def _init_state(self):
        self.s = self._z(8)

    def reset(self, mask=None):
        m = self._mask(mask)
        self.s[m] = 0.0
        self.t[m] = 0
        return self.obs()

    def obs(self):
        return self.s.clone()

    def step(self, actions):
        tq = (self._check(actions).to(self.dtype) - 1.0) * 0.5
        v = (self.s[:, 1] + tq * 0.1).clamp(-2.0, 5.0)
        self.s[:, 1] = v
        self.s[:, 0] = self.s[:, 0] + v * 0.02
        return self._finish(v - 0.1 * tq * tq, torch.zeros(self.n, dtype=torch.bool, device=self.device),
                            self.max_steps)


class ReacherLite(BatchedEnv):
    """Two-link arm with unit links: action moves joint 1 by (a - 1) 0.1; reward -|tip - target|^2,
    done when that is below 0.05; 200 steps. Obs (theta1, theta2, target_x, target_y)."""
    obs_dim, num_actions, max_steps, obs_low, obs_high = 4, 3, 200, -3.14, 3.14

    def _init_state(self):
        self.s = self._z(4)

    def reset(self, mask=None):
        m = self._mask(mask)
        self.s[m] = torch.tensor([0.0, 0.0, 0.5, 0.5], dtype=self.dtype, device=self.device)
        self.t[m] = 0
        return self.obs()

    def obs(self):
        return self.s.clone()

    def step(self, actions):
        d = (self._check(actions).to(self.dtype) - 1.0) * 0.1
        self.s[:, 0] = self.s[:, 0] + d
        t1, t2, tx, ty = self.s.unbind(1)
        ex, ey = torch.cos(t1) + torch.cos(t2), torch.sin(t1) + torch.sin(t2)
        dist = (ex - tx) ** 2 + (ey - ty) ** 2
        return self._finish(-dist, dist < 0.05, self.max_steps)


# ------------------------------------------------------------------------------------------ wrappers
def _base(env) -> BatchedEnv:
    while not isinstance(env, BatchedEnv):
        env = env.env
    return env


class FrameStack:
    """Observation = the last k observations concatenated (the reset observation repeated k times)."""

    def __init__(self, env: BatchedEnv, k: int):
        self.env, self.k = env, max(int(k), 1)
        self.n, self.num_actions, self.obs_dim = env.n, env.num_actions, env.obs_dim * self.k
        self.frames = env.obs().repeat(1, self.k)

    def reset(self, mask=None):
        o = self.env.reset(mask)
        m = _base(self.env)._mask(mask)
        self.frames[m] = o[m].repeat(1, self.k)
        return self.frames.clone()

    def step(self, actions):
        o, r, d, tr = self.env.step(actions)
        d0 = o.shape[1]
        self.frames = torch.cat([self.frames[:, d0:], o], 1)
        return self.frames.clone(), r, d, tr


class TimeLimit:
    """Truncate after max_steps steps of this wrapper (on top of the environment's own cap)."""

    def __init__(self, env, max_steps: int):
        self.env, self.max_steps = env, int(max_steps)
        self.n, self.num_actions, self.obs_dim = env.n, env.num_actions, env.obs_dim
        self.count = torch.zeros(env.n, dtype=torch.long, device=_base(env).device)

    def reset(self, mask=None):
        m = torch.ones(self.n, dtype=torch.bool, device=self.count.device) if mask is None else mask
        self.count[m] = 0
        return self.env.reset(mask)

    def step(self, actions):
        o, r, d, tr = self.env.step(actions)
        self.count += 1
        return o, r, d, tr | (self.count >= self.max_steps)


class RewardScale:
    def __init__(self, env, scale: float):
        self.env, self.scale = env, float(scale)
        self.n, self.num_actions, self.obs_dim = env.n, env.num_actions, env.obs_dim

    def reset(self, mask=None):
        return self.env.reset(mask)

    def step(self, actions):
        o, r, d, tr = self.env.step(actions)
        return o, r * self.scale, d, tr


class SingleEnv:
    """The reference's one-instance API over a batched environment of size 1."""

    def __init__(self, env):
        self.env = env
        self.num_actions, self.obs_dim = env.num_actions, env.obs_dim

    def reset(self) -> torch.Tensor:
        return self.env.reset()[0]

    def step(self, action: int) -> EnvStep:
        o, r, d, tr = self.env.step(torch.tensor([int(action)]))
        return EnvStep(o[0], float(r[0]), bool(d[0]), bool(tr[0]))

    def action_space(self) -> Space:
        return Space(n=self.num_actions)
