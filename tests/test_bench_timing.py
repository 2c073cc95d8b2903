"""The bench's timing harness (CPU, with fake CUDA events and a fake process
group): W untimed warm-up steps, then exactly K timed steps bracketed by a
barrier and a synchronize, the max over ranks, and the separate per-step pass
for the median / min / max."""
import bench


class _Clock:
    """Device time advances 1 ms per step, or the step's own duration."""

    def __init__(self, durations=None):
        self.now = 0.0
        self.steps = 0
        self.log = []
        self.durations = durations or {}

    def step(self):
        self.now += self.durations.get(self.steps, 1.0)
        self.steps += 1
        self.log.append("step")


class _Event:
    def __init__(self, clock):
        self.clock = clock
        self.t = None

    def record(self):
        self.t = self.clock.now
        self.clock.log.append("record")

    def elapsed_time(self, other):
        return other.t - self.t


class _Tensor:
    def __init__(self, v):
        self.v = v

    def item(self):
        return self.v


class _FakeTorch:
    float64 = "f64"

    def __init__(self, clock):
        clock_ = clock

        class _Cuda:
            @staticmethod
            def Event(enable_timing=True):
                return _Event(clock_)

            @staticmethod
            def synchronize():
                clock_.log.append("sync")

        self.cuda = _Cuda

    @staticmethod
    def tensor(vals, device=None, dtype=None):
        return _Tensor(vals[0])


class _FakeDist:
    class ReduceOp:
        MAX = "max"

    def __init__(self, clock, other_rank_ms):
        self.clock = clock
        self.other = other_rank_ms

    def barrier(self):
        self.clock.log.append("barrier")

    def all_reduce(self, t, op=None):
        assert op == "max"
        t.v = max(t.v, self.other)


def _timed_region(log):
    """The entries between the start and end event records of the timed region."""
    first = log.index("record")
    last = log.index("record", first + 1)
    return log[first + 1:last], log[:first], log[last + 1:]


def test_single_gpu_times_exactly_k_steps_after_w_warmups():
    clock = _Clock()
    stats = {}
    sec = bench.time_device(_FakeTorch(clock), clock.step, 3, 5, None, 1, stats=stats)
    inside, before, after = _timed_region(clock.log)
    assert inside == ["step"] * 5
    assert before.count("step") == 3 and before[-1] == "sync"
    assert abs(sec - 1e-3) < 1e-12
    assert clock.steps == 3 + 5 + 5          # warm-up, timed, per-step pass
    assert stats["reps"] == 5 and stats["median_ms"] == 1.0
    assert stats["min_ms"] == 1.0 and stats["max_ms"] == 1.0
    assert after[0] == "sync"


def test_ranks_barrier_then_sync_and_report_the_slowest():
    clock = _Clock()
    dist = _FakeDist(clock, other_rank_ms=1.5)
    sec = bench.time_device(_FakeTorch(clock), clock.step, 4, 6, dist, 2)
    inside, before, after = _timed_region(clock.log)
    assert inside == ["step"] * 6
    assert before[-2:] == ["barrier", "sync"]  # the barrier queues behind the warm-up
    assert after[:2] == ["sync", "barrier"]
    assert abs(sec - 1.5e-3) < 1e-12          # max over ranks


def test_per_step_statistics_see_a_slow_step():
    # steps are numbered from 0: 2 warm-up, 4 timed (2..5), 4 per-step (6..9)
    clock = _Clock(durations={7: 3.0})
    stats = {}
    bench.time_device(_FakeTorch(clock), clock.step, 2, 4, None, 1, stats=stats)
    assert stats["max_ms"] == 3.0 and stats["min_ms"] == 1.0 and stats["median_ms"] == 1.0
