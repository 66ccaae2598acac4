"""Randomised differential test of the page bookkeeping: seeded random sequences of prefills
(whole and partial pages), decodes (with and without the residency check), explicit evictions,
clears, layer initialisations and pool reservations over several managers and layers, replayed on
the oracle restatement (which follows the reference's scan-and-sort eviction, kv_cache.py:121-172)
and on the helm_b200 runtime (heap-ordered eviction candidates); every snapshot after every op --
page ids, states, start/used tokens, tails, free-pool order, report_usage(), bytes per tier --
must be identical.  CPU only (stand-in 'cuda' device)."""
import numpy as np
import pytest

from tests.test_bookkeeping_parity import _compare
from tests.trace_replay import replay_oracle, replay_product


def _random_spec(seed):
    rng = np.random.default_rng(seed)
    P = int(rng.choice([4, 8]))
    Hkv, D = 2, 4
    n_mgr = int(rng.integers(1, 4))
    n_layers = int(rng.integers(1, 5))
    page_bytes = 2 * Hkv * P * D * 2          # bfloat16 pages
    watermarks = [int(rng.integers(0, 12)) * page_bytes + int(rng.integers(0, 2)) * (page_bytes // 2)
                  for _ in range(n_mgr)]
    ops = []
    for _ in range(int(rng.integers(40, 90))):
        r = rng.random()
        mi = int(rng.integers(0, n_mgr))
        lid = int(rng.integers(0, n_layers))
        if r < 0.35:
            n = int(rng.choice([P, 2 * P, 3 * P + 1, int(rng.integers(1, 4 * P))]))
            ops.append(["prefill", mi, lid, n])
        elif r < 0.80:
            ops.append(["decode", mi, lid, 1, {"skip": bool(rng.random() < 0.3)}])
        elif r < 0.88:
            ops.append(["evict", mi, int(rng.integers(0, 6)) * page_bytes + int(rng.integers(0, page_bytes))])
        elif r < 0.92:
            ops.append(["clear", mi])
        elif r < 0.96:
            ops.append(["init_layers", mi, n_layers])
        else:
            ops.append(["reserve", int(rng.integers(1, 10)), "cuda" if rng.random() < 0.5 else "cpu"])
    return {"name": f"random{seed}", "seed": seed,
            "alloc": {"num_layers": n_layers, "Hkv": Hkv, "D": D, "P": P, "dtype": "bfloat16"},
            "watermarks": watermarks, "ops": ops}


@pytest.mark.parametrize("seed", range(40))
def test_runtime_matches_oracle_on_random_traces(seed):
    spec = _random_spec(seed)
    _compare(replay_product(spec), replay_oracle(spec), exact_checksums=False)


def test_random_traces_evict():
    """The generated traces do move pages to the host (and leave DEAD pages behind)."""
    moved = 0
    for seed in range(40):
        for snap in replay_oracle(_random_spec(seed)):
            moved += snap["usage"]["active_cpu_pages"] > 0
    assert moved > 100
