"""Host-side behaviour of the multi-GPU pool (tt_atom/batch.py), on CPU with toy handlers.

The reference's contract (tt_atom/batch.py:318-325, 338-380): results in input order, and a
system that fails comes back as ``{ok: False, error, tb}`` while the others still return. This
pool also survives a worker process that dies: the system it held is reported failed and the
rest run on the remaining workers. No GPU is touched: the handlers are plain Python."""
import os

import pytest

from tt_atom.batch import MultiCardSim, _DevicePool, _system_message


class Square:
    """Toy handler: squares the payload; 'boom' raises; 'die' kills the worker process."""

    def __init__(self, tag):
        self.tag = tag
        self.pid = os.getpid()

    def __call__(self, x):
        if x == "boom":
            raise ValueError("no edges within cutoff")
        if x == "die":
            os._exit(3)
        return dict(ok=True, value=x * x, pid=self.pid, tag=self.tag)


class FailsToStart:
    def __init__(self):
        raise RuntimeError("no such bundle")


def test_results_in_input_order_over_two_workers():
    with _DevicePool(Square, ("t",), device_ids=(0, 1)) as pool:
        out = pool.map(list(range(20)))
    assert [r["value"] for r in out] == [i * i for i in range(20)]
    assert len({r["pid"] for r in out}) == 2      # both workers took systems


def test_poisoned_system_fails_alone():
    with _DevicePool(Square, ("t",), device_ids=(0, 1)) as pool:
        out = pool.map([1, 2, "boom", 4, 5])
        again = pool.map([6, 7])                  # the pool keeps serving
    assert [r.get("value") for r in out] == [1, 4, None, 16, 25]
    bad = out[2]
    assert bad["ok"] is False
    assert bad["error"] == "ValueError: no edges within cutoff"
    assert "Traceback" in bad["tb"]
    assert [r["value"] for r in again] == [36, 49]


def test_dead_worker_is_reported_and_the_rest_finish():
    with _DevicePool(Square, ("t",), device_ids=(0, 1)) as pool:
        out = pool.map([1, 2, 3, "die", 5, 6, 7, 8])
        assert len(pool.live_devices) == 1
        later = pool.map([9, 10])
    assert out[3]["ok"] is False and "WorkerDied" in out[3]["error"]
    assert "exited with code 3" in out[3]["error"]
    assert [out[i]["value"] for i in (0, 1, 2, 4, 5, 6, 7)] == [1, 4, 9, 25, 36, 49, 64]
    assert [r["value"] for r in later] == [81, 100]


def test_all_workers_dead_fails_the_remaining_systems():
    with _DevicePool(Square, ("t",), device_ids=(0,)) as pool:
        out = pool.map([1, "die", 3, 4])
    assert out[0]["value"] == 1
    assert "WorkerDied" in out[1]["error"]
    assert all(r["ok"] is False and "no live worker" in r["error"] for r in out[2:])


def test_start_up_failure_raises():
    with pytest.raises(RuntimeError, match="worker failed to start: device 0: "
                                           "RuntimeError: no such bundle"):
        _DevicePool(FailsToStart, (), device_ids=(0,))


def test_sim_params_validation_and_system_messages():
    with pytest.raises(ValueError, match="mode 'relax', 'md', or 'energy'"):
        MultiCardSim("x.npz", device_ids=(0,), sim_params=dict(mode="anneal"))
    m = _system_message(([[0, 0, 0], [1, 0, 0]], [1, 1]))
    assert m["pos"].dtype.name == "float32" and m["Z"].dtype.name == "int64"
    with pytest.raises(ValueError):
        _system_message({"pos": [[0, 0, 0]]})
