"""LR schedulers (behaviour of sae_lens/training/optim.py; expected values follow
tests/training/test_optim.py) and the pure-function schedule used by the native engines."""

import pytest
import torch
from torch.optim import Adam
from torch.optim.lr_scheduler import CosineAnnealingLR, CosineAnnealingWarmRestarts

from saelens_b200.training.optim import LRSchedule, get_lr_scheduler

LR = 0.1


def _opt():
    return Adam([torch.nn.Parameter(torch.tensor(1.0))], lr=LR)


def _step(opt, sch, n=1):
    for _ in range(n):
        opt.step()
        sch.step()


def _sched(name, **kw):
    opt = _opt()
    args = dict(lr=LR, training_steps=4, warm_up_steps=0, decay_steps=0, lr_end=0.0, num_cycles=1)
    args.update(kw)
    return opt, get_lr_scheduler(name, opt, **args)


def test_unknown_scheduler():
    with pytest.raises(ValueError, match="Unsupported scheduler: unknown"):
        _sched("unknown", training_steps=10)


def test_constant():
    opt, s = _sched("constant")
    assert s.get_last_lr() == [0.1]
    _step(opt, s, 3)
    assert s.get_last_lr() == [0.1]


def test_constant_with_warmup():
    opt, s = _sched("constant", warm_up_steps=2)
    assert s.get_last_lr() == [pytest.approx(0.05)]
    _step(opt, s)
    assert s.get_last_lr() == [0.1]
    _step(opt, s, 3)
    assert s.get_last_lr() == [0.1]


def test_linear_warmup_decay():
    opt, s = _sched("constant", warm_up_steps=2, decay_steps=4, training_steps=6)
    seen = [s.get_last_lr()[0]]
    for _ in range(6):
        _step(opt, s)
        seen.append(s.get_last_lr()[0])
    assert seen == pytest.approx([0.05, 0.1, 0.1, 0.075, 0.05, 0.025, 0.0])


def test_decay_with_zero_lr_end_raises():
    with pytest.raises(ValueError, match="Cannot have decay_steps with lr_end=0.0"):
        _sched("cosineannealing", decay_steps=2, training_steps=6)


def test_cosine_annealing_main_scheduler():
    _, s = _sched("cosineannealing", lr_end=0.05)
    assert len(s._schedulers) == 1
    main = s._schedulers[0]
    assert isinstance(main, CosineAnnealingLR) and main.T_max == 4 and main.eta_min == 0.05


def test_cosine_with_warmup_and_decay_matches_plain_cosine():
    opt, s = _sched("cosineannealing", warm_up_steps=2, training_steps=8, decay_steps=2, lr_end=0.01)
    assert s.get_last_lr() == [0.05]
    _step(opt, s)
    assert s.get_last_lr() == [0.1]
    _step(opt, s)
    ref_opt = _opt()
    ref = CosineAnnealingLR(ref_opt, T_max=4, eta_min=0.01)
    for _ in range(4):
        _step(opt, s)
        _step(ref_opt, ref)
        assert s.get_last_lr() == pytest.approx(ref.get_last_lr())
    assert s.get_last_lr() == [pytest.approx(0.01)]


def test_cosine_warm_restarts():
    _, s = _sched("cosineannealingwarmrestarts", training_steps=8, lr_end=0.05, num_cycles=2)
    main = s._schedulers[0]
    assert isinstance(main, CosineAnnealingWarmRestarts) and main.T_0 == 4 and main.eta_min == 0.05


@pytest.mark.parametrize("name,warm,decay,cycles", [("constant", 3, 5, 1), ("cosineannealing", 4, 6, 1),
                                                    ("cosineannealingwarmrestarts", 2, 4, 3), ("constant", 0, 0, 1)])
def test_pure_schedule_matches_torch_chain(name, warm, decay, cycles):
    steps = 30
    opt, s = _sched(name, training_steps=steps, warm_up_steps=warm, decay_steps=decay, lr_end=0.01,
                    num_cycles=cycles)
    pure = LRSchedule(name, steps, LR, warm, decay, 0.01, cycles)
    for i in range(steps):
        assert pure.lr_at(i) == pytest.approx(s.get_last_lr()[0], abs=1e-7)
        _step(opt, s)
