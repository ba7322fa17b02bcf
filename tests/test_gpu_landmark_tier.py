"""The landmark bank with its members' master copies in pinned host memory (the
reference's tiered store, longctx/inference/landmark_cache_v2.py:137-411):
direct mode and the staged hot set assemble byte-identical caches and make the
same decisions as the device-resident bank, the oracle and the reference."""
import numpy as np
import pytest
import torch

import inputs as gi
from oracle import landmark as olm
from oracle.numerics import torch_bf16_to_bits

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("hot", [0, 2, 5])
def test_host_tier_stack_matches_oracle_without_host_syncs(cuda, hot):
    """Many chunks queued back to back (no host synchronisation between them): every
    layer's assembled cache equals the chunks the oracle's layout names."""
    from reworld_b200 import _native
    from reworld_b200.landmark import LandmarkBankStack
    from reworld_b200.poses import random_walk
    ct, H, D, L = 8, 2, 128, 3
    poses = random_walk(40, seed=11, revisit_every=6)
    st = LandmarkBankStack(ct, L, H, D, n_sink=1, recent_w=3, K=6, retrieve_k=2, device=cuda, host_tier=True,
                           hot_gpu=hot, gpu_spare=1)
    ob = olm.OracleBank(1, 3, 6, 2, "b")
    gen = torch.Generator(device=cuda).manual_seed(12)
    data, snaps, layouts = {}, [], []
    caps = [torch.zeros(1, 8 * ct, H, D, dtype=torch.bfloat16, device=cuda) for _ in range(2 * L)]
    for c in range(len(poses) - 1):
        kvs = torch.randn(L, 2, ct, H, D, generator=gen, device=cuda).to(torch.bfloat16)
        data[c] = kvs
        R = st.add_chunk_from([kvs[l, 0] for l in range(L)], [kvs[l, 1] for l in range(L)], poses[c], poses[c + 1])
        assert R == ob.add_chunk(poses[c], poses[c + 1]), f"retrieval differs at chunk {c}"
        tot = st.write_into_caches(caps[:L], caps[L:], R)
        lay = ob.layout(R)
        assert tot == len(lay) * ct
        snaps.append([cp[0, :tot].clone() for cp in caps])   # ordered on the compute stream
        layouts.append(lay)
    torch.cuda.synchronize()
    for c, (snap, lay) in enumerate(zip(snaps, layouts)):
        for l in range(L):
            assert torch.equal(snap[l], torch.cat([data[b][l, 0] for b in lay])), (c, l)
            assert torch.equal(snap[L + l], torch.cat([data[b][l, 1] for b in lay])), (c, l)
    s = st.stats([0, 1])
    assert s["host_slots_used"] == len(st.bank) <= 6 and s["io_bytes_d2h"] > 0 and s["io_bytes_h2d"] > 0
    if hot:
        assert s["hot"] <= max(hot, 2) and s["io_misses"] > 0
    _native.check_status(cuda)


@pytest.mark.parametrize("hot_gpu", [None, 4])
@pytest.mark.parametrize("name", gi.landmark_runs_names()[:3])
def test_host_tier_drop_in_vs_reference(cuda, golden, name, hot_gpu):
    """LandmarkCacheV2(host_tier=True): the reference's retrieval, bank contents and
    write_into_cache bytes, chunk by chunk."""
    from reworld_b200.landmark import LandmarkCacheV2
    g = golden["landmark"]
    poses, ct, H, D, ns, rw, K, rk, mode = gi.landmark_runs()[name]
    lm = LandmarkCacheV2(ct, n_sink=ns, recent_w=rw, K=K, retrieve_k=rk, mode=mode, host_tier=True,
                         hot_gpu=hot_gpu)
    N = len(poses) - 1
    cap = (ns + rw + (K if mode == "a" else rk)) * ct + 4
    tail = g[f"{name}_cache_tail"]
    for c in range(N):
        k, v = gi.landmark_kv(name, c, ct, H, D)
        R = lm.add_chunk(k.to(cuda), v.to(cuda), poses[c], poses[c + 1])
        assert R == [int(x) for x in g[f"{name}_R"][c] if x >= 0], f"retrieval differs at chunk {c}"
        assert [e.born for e in lm.bank] == [int(x) for x in g[f"{name}_bank"][c] if x >= 0]
        kc = {"k": torch.zeros(1, cap, H, D, dtype=torch.bfloat16, device=cuda),
              "v": torch.zeros(1, cap, H, D, dtype=torch.bfloat16, device=cuda)}
        tot = lm.write_into_cache(kc, R)
        assert tot == int(g[f"{name}_tot"][c])
        if c >= N - 3:
            t = c - (N - 3)
            assert np.array_equal(torch_bf16_to_bits(kc["k"]), tail[t, 0])
            assert np.array_equal(torch_bf16_to_bits(kc["v"]), tail[t, 1])
            k2, v2, tot2 = lm.get_active_kv(R)
            assert tot2 == tot and torch.equal(k2, kc["k"][0, :tot]) and torch.equal(v2, kc["v"][0, :tot])


def test_host_tier_refuses_a_pool_smaller_than_the_retrieved_landmarks(cuda, monkeypatch):
    """A host pool capped below retrieve_k (little pinnable memory) cannot hold the
    landmarks a chunk retrieves: the bank refuses it instead of running short."""
    from reworld_b200 import landmark as lm
    real_pool = lm.host_pool
    monkeypatch.setattr(lm, "host_pool", lambda n, shape, dtype: real_pool(min(n, 2), shape, dtype))
    with pytest.raises(RuntimeError, match="fewer than the 3 landmarks"):
        lm.LandmarkBankStack(8, 2, 2, 128, n_sink=1, recent_w=3, K=6, retrieve_k=3, device=cuda,
                             host_tier=True)
    # a pool of at least retrieve_k members is accepted, with K lowered to it
    monkeypatch.setattr(lm, "host_pool", lambda n, shape, dtype: real_pool(min(n, 3), shape, dtype))
    st = lm.LandmarkBankStack(8, 2, 2, 128, n_sink=1, recent_w=3, K=6, retrieve_k=3, device=cuda,
                              host_tier=True)
    assert st.K == 3
