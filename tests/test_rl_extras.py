"""Batched RL environments against one-instance loops that restate the reference's dynamics
(crates/brain-rl/src/env/gym.rs, atari_lite.rs, mujoco_lite.rs, wrappers.rs), and the buffers,
distributions, value functions, skill library, agents, trainers and checkpoints of
crates/brain-rl/src (buffer/sequence.rs, policy/dist.rs, value/qvalue.rs, skill_library.rs, dqn/,
trainer.rs, eval.rs, checkpoint.rs, utils.rs)."""
import math

import pytest
import torch

from brain_b200.zoo import rl_agents as RA
from brain_b200.zoo import rl_envs as E
from brain_b200.zoo.rl import DqnConfig, Transition


def _cartpole_ref(state, a):
    x, xd, th, thd = state
    force = 10.0 if a == 1 else -10.0
    c, s = math.cos(th), math.sin(th)
    total, pml = 1.1, 0.05
    temp = (force + pml * thd * thd * s) / total
    thacc = (9.8 * s - c * temp) / (0.5 * (4.0 / 3.0 - 0.1 * c * c / total))
    xacc = temp - pml * thacc * c / total
    x, xd, th, thd = x + 0.02 * xd, xd + 0.02 * xacc, th + 0.02 * thd, thd + 0.02 * thacc
    lim = 12 * 2 * math.pi / 360
    return [x, xd, th, thd], 1.0, x < -2.4 or x > 2.4 or th < -lim or th > lim


def _mountain_ref(state, a):
    p, v = state
    v = min(max(v + (a - 1) * 0.001 + math.cos(3 * p) * -0.0025, -0.07), 0.07)
    p = min(max(p + v, -1.2), 0.6)
    if p <= -1.2 and v < 0:
        v = 0.0
    return [p, v], -1.0, p >= 0.5


def _pong_ref(state, a):
    py, bx, by, vx, vy = state
    if a == 1:
        py = max(py - 0.05, 0.0)
    elif a == 2:
        py = min(py + 0.05, 1.0)
    bx, by = bx + vx, by + vy
    if by <= 0 or by >= 1:
        vy = -vy
    r, d = 0.0, False
    if bx >= 1:
        vx = -vx
    if bx <= 0:
        if abs(by - py) < 0.15:
            r, vx = 1.0, -vx
        else:
            r, d = -1.0, True
    return [py, bx, by, vx, vy], r, d


@pytest.mark.parametrize("cls,ref,init", [(E.CartPole, _cartpole_ref, [0.0, 0, 0, 0]),
                                          (E.MountainCar, _mountain_ref, [-0.5, 0.0]),
                                          (E.PongLite, _pong_ref, [0.5, 0.5, 0.5, 0.05, 0.03])])
def test_batched_envs_match_reference_dynamics(cls, ref, init):
    n = 5
    env = cls(n)
    g = torch.Generator().manual_seed(3)
    states = [list(init) for _ in range(n)]
    steps = [0] * n
    for _ in range(300):
        a = torch.randint(0, env.num_actions, (n,), generator=g)
        obs, r, d, tr = env.step(a)
        for i in range(n):
            states[i], ri, di = ref(states[i], int(a[i]))
            steps[i] += 1
            assert float(r[i]) == pytest.approx(ri) and bool(d[i]) == di
            assert bool(tr[i]) == (steps[i] >= env.max_steps)
            want = states[i] if cls is not E.PongLite else states[i]
            torch.testing.assert_close(obs[i], torch.tensor(want, dtype=torch.float64)[:env.obs_dim], rtol=1e-12,
                                       atol=1e-12)
        end = d | tr
        if bool(end.any()):
            env.reset(end)
            for i in range(n):
                if bool(end[i]):
                    states[i], steps[i] = list(init), 0
    with pytest.raises(ValueError):
        env.step(torch.full((n,), env.num_actions))


def test_other_envs_and_wrappers():
    p = E.Pendulum(2)
    o, r, d, tr = p.step(torch.tensor([2, 0]))
    thd = min(max(0 + (-15.0 * math.sin(math.pi) + 3.0 * 2.0) * 0.05, -8), 8)
    assert float(o[0, 2]) == pytest.approx(thd) and float(r[0]) == pytest.approx(-((thd * 0.05) ** 2 + 0.1 * thd ** 2 + 0.004))
    assert not bool(d.any())
    hc = E.HalfCheetahLite(1)
    _, r, _, _ = hc.step(torch.tensor([2]))
    assert float(r[0]) == pytest.approx(0.05 - 0.1 * 0.25) and float(hc.s[0, 0]) == pytest.approx(0.05 * 0.02)
    re = E.ReacherLite(1)
    o, r, d, _ = re.step(torch.tensor([2]))
    ex, ey = math.cos(0.1) + 1.0, math.sin(0.1)
    assert float(r[0]) == pytest.approx(-((ex - 0.5) ** 2 + (ey - 0.5) ** 2))
    br = E.BreakoutLite(3)
    for _ in range(10):
        o, r, d, tr = br.step(torch.tensor([0, 1, 2]))
    assert o.shape == (3, 3)
    fs = E.FrameStack(E.CartPole(2), 3)
    o0 = fs.reset()
    assert o0.shape == (2, 12) and torch.equal(o0[:, :4], o0[:, 8:])
    o1, *_ = fs.step(torch.tensor([1, 0]))
    assert torch.equal(o1[:, :8], o0[:, 4:])
    tl = E.TimeLimit(E.RewardScale(E.Pendulum(2), 0.5), 3)
    tl.reset()
    for i in range(3):
        _, r, _, tr = tl.step(torch.tensor([1, 1]))
    assert bool(tr.all()) and float(r[0]) <= 0.0
    single = E.SingleEnv(E.MountainCar(1))
    assert single.reset().tolist() == [-0.5, 0.0]
    st = single.step(2)
    assert isinstance(st, E.EnvStep) and st.reward == -1.0 and not st.done


def test_buffers_dists_values_skills():
    nb = RA.NStepBuffer(3, 0.9)
    z = torch.zeros(2)
    outs = [nb.push(Transition(z + i, i, float(i + 1), z + i + 1, i == 3)) for i in range(5)]
    assert outs[0] is None and outs[1] is None
    assert outs[2].reward == pytest.approx(1 + 0.9 * 2 + 0.81 * 3) and outs[2].action == 0 and not outs[2].done
    assert outs[3].reward == pytest.approx(2 + 0.9 * 3 + 0.81 * 4) and outs[3].done  # stops at the done step
    cd = RA.CategoricalDist.from_logits([1.0, 2.0, 3.0])
    p = torch.softmax(torch.tensor([1.0, 2.0, 3.0], dtype=torch.float64), 0)
    assert cd.log_prob(2) == pytest.approx(math.log(float(p[2]))) and cd.log_prob(7) == -1e10
    assert cd.entropy() == pytest.approx(float(-(p * p.log()).sum()))
    gd = RA.DiagonalGaussianDist([0.0, 1.0], [0.0, math.log(2.0)])
    want = sum(-0.5 * ((a - m) ** 2 / s ** 2 + math.log(2 * math.pi * s ** 2)) for a, m, s in ((0.5, 0, 1), (0, 1, 2)))
    assert gd.log_prob([0.5, 0.0]) == pytest.approx(want)
    assert gd.entropy() == pytest.approx(2 * (0.5 + 0.5 * math.log(2 * math.pi)) + math.log(2.0))
    assert RA.GaussianPolicy(2).distribution([0.0, 0.0]).entropy() == pytest.approx(1 + math.log(2 * math.pi))
    qt = RA.QTable()
    qt.update_q(0, 1, 1.0, 1, 2, 0.9, 0.5)
    assert qt.get(0, 1) == 0.5 and qt.max_q(5, 3) == 0.0
    qn = RA.QNet(3, 2)
    assert qn(torch.ones(4, 3)).shape == (4, 2)
    lib = RA.SkillLibrary()
    lib.insert(RA.Skill("walk", [1.0, 0.0]))
    lib.insert(RA.Skill("jump", [0.0, 1.0]))
    lib.insert(RA.Skill("walk", [1.0, 0.0], cumulative_reward=3.0))
    assert len(lib) == 2 and lib.skills[0].success_count == 1 and lib.skills[0].cumulative_reward == 3.0
    assert lib.search([0.9, 0.1], 0.5).name == "walk" and lib.search([1.0, 1.0], 0.8) is None
    assert lib.search([1.0], 0.0) is None  # length mismatch -> similarity 0, not above the floor
    torch.testing.assert_close(RA.discount_returns([1.0, 1.0, 1.0], 0.5), torch.tensor([1.75, 1.5, 1.0], dtype=torch.float64))
    assert RA.moving_average([1.0, 3.0, 5.0], 0.5) == [1.0, 2.0, 3.5]


def test_agents_trainers_eval_checkpoint():
    cfg = DqnConfig(batch_size=16, buffer_capacity=500, target_update=20, epsilon_decay_steps=100, hidden=32)
    env = E.SingleEnv(E.CartPole(1))
    agent = RA.DoubleDqnAgent(4, 2, cfg, seed=1)
    rewards = RA.DqnTrainer(agent, env, RA.TrainerConfig(max_episodes=4, max_steps_per_episode=60)).train()
    assert len(rewards) == 4 and all(r >= 1 for r in rewards)
    rep = RA.evaluate_dqn(agent, env, 3)
    assert rep.num_episodes == 3 and rep.min_return <= rep.mean_return <= rep.max_return
    with pytest.raises(ValueError):
        RA.evaluate_dqn(agent, env, 0)
    ck = RA.RlCheckpoint.save_dqn(agent)
    other = RA.DoubleDqnAgent(4, 2, cfg, seed=2)
    ck.load_dqn(other)
    assert other.total_steps == agent.total_steps
    assert torch.equal(other.q_online.weight, agent.q_online.weight)
    with pytest.raises(ValueError):
        ck.load_dqn(RA.DoubleDqnAgent(5, 2, cfg))
    rb = RA.RainbowAgent(4, 2, cfg, n_steps=3, seed=0)
    losses = RA.DqnTrainer(rb, env, RA.TrainerConfig(max_episodes=3, max_steps_per_episode=40)).train()
    assert len(losses) == 3 and len(rb.per_buffer) > 0


def test_batched_dqn_trainer_runs_many_instances():
    env = E.CartPole(32)
    tr = RA.BatchedDqnTrainer(env, hidden=32, capacity=4096, batch_size=64, eps_decay_steps=50, seed=0)
    losses = [tr.step() for _ in range(120)]
    assert all(math.isfinite(v) for v in losses) and len(tr.finished) > 0
    assert tr.size == min(120 * 32, 4096)
