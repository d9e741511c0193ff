"""Test stand-in for the part of Optuna's interface that the reference's
engine calls (bo_kernel_tuner/tuner/engine.py: create_study, enqueue_trial,
optimize with callbacks and catch, TrialPruned, TrialState, Grid/Random
samplers).  Optuna is not installed in this image; this lets the drop-in tests
run the reference's unmodified run_search / run_benchmark over the sm_100a
kernels.  Grid order is a seeded shuffle without repetition and the study stops
when the grid is exhausted, as Optuna's GridSampler does; random draws are
seeded.  There is no TPE here: constructing TPESampler raises."""

import enum
import itertools
import random
import time
import types


class TrialPruned(Exception):
    pass


class TrialState(enum.Enum):
    RUNNING = 0
    COMPLETE = 1
    PRUNED = 2
    FAIL = 3
    WAITING = 4


trial = types.SimpleNamespace(TrialState=TrialState)


class GridSampler:
    def __init__(self, space, seed=None):
        names = list(space)
        self.points = [dict(zip(names, v)) for v in itertools.product(*space.values())]
        random.Random(seed).shuffle(self.points)
        self.next = 0

    def draw(self, study):
        if self.next >= len(self.points):
            return None
        p = self.points[self.next]
        self.next += 1
        if self.next >= len(self.points):
            study.stop()
        return p


class RandomSampler:
    def __init__(self, seed=None):
        self.rng = random.Random(seed)

    def draw(self, study):
        return None  # values are drawn in suggest_categorical


class TPESampler:
    def __init__(self, *args, **kwargs):
        raise RuntimeError("TPE is not available in the test stand-in for optuna")


samplers = types.SimpleNamespace(GridSampler=GridSampler, RandomSampler=RandomSampler,
                                 TPESampler=TPESampler)


class FrozenTrial:
    def __init__(self, number, params, user_attrs):
        self.number = number
        self.params = dict(params)
        self.user_attrs = dict(user_attrs)
        self.state = TrialState.RUNNING
        self.value = None


class Trial:
    def __init__(self, frozen, fixed, rng):
        self._frozen = frozen
        self._fixed = fixed or {}
        self._rng = rng
        self.number = frozen.number

    def suggest_categorical(self, name, choices):
        value = self._fixed[name] if name in self._fixed else self._rng.choice(list(choices))
        self._frozen.params[name] = value
        return value

    def set_user_attr(self, key, value):
        self._frozen.user_attrs[key] = value


class Study:
    def __init__(self, sampler):
        self.sampler = sampler
        self.trials = []
        self.user_attrs = {}
        self._queue = []
        self._stop = False
        self._rng = getattr(sampler, "rng", random.Random(0))

    def set_user_attr(self, key, value):
        self.user_attrs[key] = value

    def enqueue_trial(self, params, user_attrs=None):
        self._queue.append((dict(params), dict(user_attrs or {})))

    def stop(self):
        self._stop = True

    def optimize(self, objective, n_trials=None, timeout=None, n_jobs=1, catch=(),
                 callbacks=()):
        start = time.perf_counter()
        done = 0
        while (n_trials is None or done < n_trials) and not self._stop:
            if timeout is not None and time.perf_counter() - start >= timeout:
                break
            if self._queue:
                fixed, attrs = self._queue.pop(0)
            else:
                fixed, attrs = self.sampler.draw(self), {}
                if fixed is None and isinstance(self.sampler, GridSampler):
                    break
            frozen = FrozenTrial(len(self.trials), {}, attrs)
            self.trials.append(frozen)
            try:
                frozen.value = objective(Trial(frozen, fixed, self._rng))
                frozen.state = TrialState.COMPLETE
            except TrialPruned:
                frozen.state = TrialState.PRUNED
            except Exception as exc:
                frozen.state = TrialState.FAIL
                if not isinstance(exc, tuple(catch)):
                    raise
            done += 1
            for cb in callbacks:
                cb(self, frozen)


def create_study(direction="minimize", sampler=None, study_name=None, storage=None):
    return Study(sampler or RandomSampler())
