"""Bit-exact page bookkeeping: the reference's recorded traces vs the oracle restatement and vs
the helm_b200 runtime classes (CPU; a stand-in 'cuda' device makes eviction run without a GPU).

Compared after every op: page ids, layer ids, start/used tokens, capacities, states, device
types, tails, total tokens, free-pool id order, next page id, report_usage() and
report_bytes_per_tier().  Page data is compared through per-page checksums."""
import json
import math
import pathlib

import pytest

from tests.trace_replay import replay_oracle, replay_product, split_checksums

TRACES = json.loads((pathlib.Path(__file__).resolve().parent / "golden" / "bookkeeping_traces.json").read_text())
IDS = [t["spec"]["name"] for t in TRACES]


def _compare(snaps, golden, exact_checksums: bool):
    assert len(snaps) == len(golden)
    for i, (s, g) in enumerate(zip(snaps, golden)):
        s0, sck = split_checksums(s)
        g0, gck = split_checksums(g)
        assert s0 == g0, f"op {i}: bookkeeping differs"
        for a, b in zip(sck, gck):
            assert (a is None) == (b is None), f"op {i}: DEAD page mismatch"
            if a is None:
                continue
            for x, y in zip(a, b):
                if exact_checksums:
                    assert x == y, f"op {i}: page data checksum {x} != {y}"
                else:
                    assert math.isclose(x, y, rel_tol=1e-9, abs_tol=1e-9), f"op {i}: checksum {x} vs {y}"


@pytest.mark.parametrize("trace", TRACES, ids=IDS)
def test_oracle_matches_reference_trace(trace):
    _compare(replay_oracle(trace["spec"]), trace["snapshots"], exact_checksums=False)


@pytest.mark.parametrize("trace", TRACES, ids=IDS)
def test_runtime_matches_reference_trace(trace):
    _compare(replay_product(trace["spec"]), trace["snapshots"], exact_checksums=True)


def test_traces_exercise_eviction():
    """The fixtures must actually contain evictions, DEAD pages and non-prefix evictions."""
    dead = cpu_in_layer = mid_gpu = 0
    for t in TRACES:
        for snap in t["snapshots"]:
            for m in snap["managers"]:
                for L in m["layers"].values():
                    states = [p[5] for p in L["pages"]]
                    cpu_in_layer += states.count("CPU")
                    for i in range(1, len(states) - 1):
                        if states[i] == "GPU" and "CPU" in states[i + 1:]:
                            mid_gpu += 1
            dead += snap["usage"]["gpu_pool_size"] < snap["next_page_id"]
    assert cpu_in_layer > 0 and mid_gpu > 0 and dead > 0
