"""The rollout-side pieces around the bank (rows a12, a13): the compressed
pipeline's budget split (pipeline/causal_diffusion_inference_compressed.py:
273-282, 302-322) and its chunk pose (:355-377), against the reference's own
methods run by tests/golden/make_golden.py (pipeline.npz)."""
import os

import numpy as np
import pytest
import torch

import inputs as gi
from oracle import landmark as olm

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "pipeline.npz"))
POLICIES = gi.POLICIES


def _cases():
    for row in GOLD["budget"]:
        yield [int(x) for x in row]


def test_budget_split_matches_reference_pipeline():
    from reworld_b200.landmark import budget_split
    n = 0
    for pol, budget, n_sink, recent_w, landmark_k, cap, ct, r_sink, r_recent, r_K, r_k, r_mode_b, r_div in _cases():
        sp = budget_split(budget, n_sink, recent_w, landmark_k, POLICIES[pol],
                          cache_tokens=cap * ct if cap else None, chunk_tokens=ct)
        got = (sp.n_sink, sp.recent_w, sp.K, sp.n_landmark, int(sp.mode == "b"), int(sp.diverse))
        assert got == (r_sink, r_recent, r_K, r_k, r_mode_b, r_div), (POLICIES[pol], budget, got)
        assert sp.budget == (min(budget, cap) if cap else budget)
        n += 1
    assert n >= 12


def test_oracle_budget_split_agrees_for_top_k_policies():
    for pol, budget, n_sink, recent_w, landmark_k, cap, ct, r_sink, r_recent, r_K, r_k, r_mode_b, _ in _cases():
        if not r_mode_b or cap:
            continue
        assert olm.budget_split(budget, n_sink, recent_w, landmark_k) == (r_sink, r_recent, r_k, r_K)


def test_budget_split_refuses_other_policies():
    from reworld_b200.landmark import budget_split
    for pol in ("merge", "window", "naive", "select"):
        with pytest.raises(ValueError):
            budget_split(12, 1, 5, 30, pol)
    with pytest.raises(ValueError):
        budget_split(12, 1, 5, 30, "v15b", cache_tokens=100)


@pytest.mark.parametrize("i", range(6))
def test_chunk_pose_bit_exact(i):
    from reworld_b200.landmark import chunk_pose
    T, fpc, dt = gi.POSE_CASES[i]
    ctx = torch.from_numpy(GOLD[f"pose{i}_ctx"]).to(getattr(torch, dt))
    got = chunk_pose(ctx, fpc)
    want = GOLD[f"pose{i}_out"]
    assert got.dtype == np.float32 and got.shape == (4, 4)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (got, want)


def test_chunk_pose_needs_context():
    from reworld_b200.landmark import chunk_pose
    with pytest.raises(RuntimeError):
        chunk_pose(None, 3)


def test_bank_stack_from_budget_uses_the_split():
    from reworld_b200.landmark import LandmarkBankStack
    st = LandmarkBankStack.from_budget(8, 2, 2, 16, budget_chunks=24, n_sink=1, recent_w=7, landmark_k=120,
                                       device="cpu")
    assert (st.n_sink, st.recent_w, st.retrieve_k, st.K, st.mode) == (1, 7, 16, 120, "b")
    assert st.pool.pool.shape[0] == 1 + 7 + 120 + 1          # sink + recent + bank + the chunk being packed
    st_a = LandmarkBankStack.from_budget(8, 1, 1, 16, budget_chunks=12, policy="consol", device="cpu")
    assert (st_a.retrieve_k, st_a.K, st_a.mode) == (6, 6, "a")
