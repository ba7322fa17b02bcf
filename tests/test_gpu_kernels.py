"""RoPE + cache store, landmark gather (bulk copies), bank decisions and the
Ulysses layout transforms on the GPU, against the oracle and the reference's
fixtures.  Integer / byte / index results are compared bit for bit."""
import ctypes

import numpy as np
import pytest
import torch

import inputs as gi
from oracle import landmark as olm
from oracle import rope as orope
from oracle import ulysses as ou
from oracle.numerics import f32_to_bf16_bits, torch_bf16_to_bits

pytestmark = pytest.mark.gpu


def _status_clean():
    from reworld_b200 import _native
    _native.check_status()


@pytest.mark.parametrize("sf", [0, 7, 33])
def test_rope_store_bit_exact_vs_reference_fixture(cuda, golden, sf):
    """K roped into the cache reproduces the reference's causal_rope_apply bits."""
    from reworld_b200 import RopeArgs, device_table, rope_kv_store
    x, grid, delta = gi.rope_case()
    L, H = x.shape[1], x.shape[2]
    freqs = orope.build_freqs(128, gi.ROPE_SCALE_H, gi.ROPE_SCALE_W)
    cache_k = torch.zeros(1, L + 10, H, 128, dtype=torch.bfloat16, device=cuda)
    cache_v = torch.zeros_like(cache_k)
    v = torch.randn(1, L, H, 128).to(torch.bfloat16)
    q_out = rope_kv_store(x.to(cuda), v.to(cuda), cache_k, cache_v, 5,
                          rope=RopeArgs(device_table(freqs, cuda), grid, sf), q=x.to(cuda))
    torch.cuda.synchronize()
    want = golden["rope"][f"rope_sf{sf}"].reshape(1, L, H, 128)
    assert np.array_equal(torch_bf16_to_bits(cache_k[:, 5:5 + L]), want)
    assert np.array_equal(torch_bf16_to_bits(q_out), want)
    assert torch.equal(cache_v[:, 5:5 + L].cpu(), v)
    assert not cache_k[:, :5].any() and not cache_k[:, 5 + L:].any()
    _status_clean()


def test_rope_store_with_pm_delta_vs_reference_fixture(cuda, golden):
    from reworld_b200 import RopeArgs, device_table, rope_kv_store
    x, (f, h, w), delta = gi.rope_case()
    L, H = x.shape[1], x.shape[2]
    freqs = orope.build_freqs(128, gi.ROPE_SCALE_H, gi.ROPE_SCALE_W)
    # The pipeline's phase is per frame (pose_mlp of the frame's pose, broadcast
    # over the frame's tokens, action_model.py:171-192); the kernel takes it per
    # frame.  Compare against the oracle fed the same phase broadcast per token.
    dframe = delta[:, ::h * w][:, :f, 0]                         # [1, f, 64]
    dtok = dframe.unsqueeze(2).expand(-1, -1, h * w, -1).reshape(1, f * h * w, 1, 64)
    dtok = torch.cat([dtok, torch.zeros(1, L - f * h * w, 1, 64)], dim=1)
    y = orope.causal_rope_apply(x.float().numpy(), [(f, h, w)], freqs, start_frame=7)
    yd = orope.pm_rope_delta_apply(y, dtok.numpy())
    yd[:, f * h * w:] = x.float().numpy()[:, f * h * w:]        # tokens past the grid stay unchanged
    cache_k = torch.zeros(1, L, H, 128, dtype=torch.bfloat16, device=cuda)
    cache_v = torch.zeros_like(cache_k)
    rope_kv_store(x.to(cuda), x.to(cuda), cache_k, cache_v, 0,
                  rope=RopeArgs(device_table(freqs, cuda), (f, h, w), 7, delta=dframe.to(cuda)))
    torch.cuda.synchronize()
    # complex64 products are formed without contraction, like the CPU reference
    assert np.array_equal(torch_bf16_to_bits(cache_k), f32_to_bf16_bits(yd))


def test_copy_chunks_bit_exact_many_jobs(cuda):
    from reworld_b200.landmark import copy_jobs
    g = torch.Generator(device=cuda).manual_seed(0)
    src = torch.randint(-30000, 30000, (3_000_000,), generator=g, device=cuda, dtype=torch.int16)
    dst = torch.zeros(3_100_000, dtype=torch.int16, device=cuda)
    rng = np.random.default_rng(0)
    jobs, off_d = [], 0
    expect = torch.zeros_like(dst)
    for _ in range(57):
        nb = int(rng.integers(1, 4000)) * 16                 # 16-byte multiples, odd piece tails
        so = int(rng.integers(0, (src.numel() * 2 - nb) // 16)) * 16
        jobs.append((src.data_ptr() + so, dst.data_ptr() + off_d, nb))
        expect[off_d // 2:(off_d + nb) // 2] = src[so // 2:(so + nb) // 2]
        off_d += nb
    big = 40 * 16384 + 48                                     # one job spanning many pieces
    jobs.append((src.data_ptr(), dst.data_ptr() + off_d, big))
    expect[off_d // 2:(off_d + big) // 2] = src[:big // 2]
    copy_jobs(jobs, cuda)
    torch.cuda.synchronize()
    assert torch.equal(dst, expect)
    _status_clean()


def test_copy_chunks_flags_bad_descriptor(cuda):
    """A misaligned job is skipped and reported, the others still run."""
    from reworld_b200 import _native
    from reworld_b200.landmark import copy_jobs
    src = torch.arange(4096, dtype=torch.int16, device=cuda)
    dst = torch.zeros(4096, dtype=torch.int16, device=cuda)
    copy_jobs([(src.data_ptr(), dst.data_ptr(), 1024), (src.data_ptr() + 2, dst.data_ptr() + 2048, 32)], cuda)
    torch.cuda.synchronize()
    assert torch.equal(dst[:512], src[:512]) and not dst[512:].any()
    with pytest.raises(RuntimeError, match="out of range"):
        _native.check_status()


@pytest.mark.parametrize("name", gi.landmark_runs_names())
def test_bank_decisions_and_cache_bytes_vs_reference(cuda, golden, name):
    """Device bank (LandmarkCacheV2 drop-in): retrieved indices, bank contents,
    events and write_into_cache bytes equal the reference's, chunk by chunk."""
    from reworld_b200.landmark import LandmarkCacheV2
    g = golden["landmark"]
    poses, ct, H, D, ns, rw, K, rk, mode = gi.landmark_runs()[name]
    lm = LandmarkCacheV2(ct, n_sink=ns, recent_w=rw, K=K, retrieve_k=rk, mode=mode)
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
    ev = [(0 if e[0] == "add" else 1, e[1]) for e in lm.events]
    assert ev == [tuple(int(x) for x in e) for e in g[f"{name}_events"]]
    _status_clean()


@pytest.mark.parametrize("prepared", [False, True])
def test_bank_stack_all_layers_one_launch(cuda, prepared):
    """The all-layers stack makes the same decisions as the oracle and assembles
    every layer's cache from that layer's own chunk K/V — also when each chunk's
    decision is queued by prepare() before its K/V exist (as the rollout does,
    ahead of the chunk's forwards)."""
    from reworld_b200.landmark import LandmarkBankStack
    from reworld_b200.poses import random_walk
    ct, H, D, L = 4, 2, 128, 5
    poses = random_walk(30, seed=3, revisit_every=8)
    st = LandmarkBankStack(ct, L, H, D, n_sink=1, recent_w=3, K=6, retrieve_k=2, device=cuda)
    ob = olm.OracleBank(1, 3, 6, 2, "b")
    gen = torch.Generator(device=cuda).manual_seed(4)
    data = {}
    caps = [torch.zeros(1, 8 * ct, H, D, dtype=torch.bfloat16, device=cuda) for _ in range(2 * L)]
    for c in range(len(poses) - 1):
        if prepared:
            st.prepare(poses[c], poses[c + 1])
        kvs = torch.randn(L, 2, ct, H, D, generator=gen, device=cuda).to(torch.bfloat16)
        data[c] = kvs
        R = st.add_chunk_from([kvs[l, 0] for l in range(L)], [kvs[l, 1] for l in range(L)], poses[c], poses[c + 1])
        Ro = ob.add_chunk(poses[c], poses[c + 1])
        assert R == Ro
        tot = st.write_into_caches(caps[:L], caps[L:], R)
        lay = ob.layout(R)
        assert tot == len(lay) * ct
        for l in range(L):
            want_k = torch.cat([data[b][l, 0] for b in lay])
            want_v = torch.cat([data[b][l, 1] for b in lay])
            assert torch.equal(caps[l][0, :tot], want_k) and torch.equal(caps[L + l][0, :tot], want_v)
    if prepared:
        st.prepare(poses[0], poses[1])
        with pytest.raises(RuntimeError):   # a decision prepared for other poses is refused
            st.add_chunk_from([kvs[l, 0] for l in range(L)], [kvs[l, 1] for l in range(L)], poses[2], poses[3])
    _status_clean()


def test_bank_exact_tie_picks_lower_index(cuda):
    """All members at the same pose: every distance ties; the device takes the
    lowest bank indices (a valid top-k set; the reference's numpy argsort is
    not stable, so its choice among exact ties is implementation-defined)."""
    from reworld_b200.landmark import DeviceBankDecisions
    p = np.eye(4, dtype=np.float32)
    dec = DeviceBankDecisions(K=10, retrieve_k=3, device=cuda)
    for i in range(8):
        _, R, _ = dec.step(admit=(p, i, i), target=p)
    assert R == [0, 1, 2]


def test_bank_protected_degenerate_and_mode_a(cuda):
    from reworld_b200.landmark import DeviceBankDecisions
    from reworld_b200.poses import yaw_walk
    poses = yaw_walk(12, seed=9)
    # protect_n >= K: eviction falls back to all members (reference warning branch)
    dec = DeviceBankDecisions(K=2, retrieve_k=1, protect_n=2, device=cuda)
    ob = olm.OracleBank(0, 0, 2, 1, "b", protect_n=2)
    for i in range(10):
        ev, R, _ = dec.step(admit=(poses[i], i, i), target=poses[i + 1])
        ob.poses[i] = poses[i]
        ob._bank_insert(i)
        assert R == ob._retrieve(poses[i + 1])
        assert [m[0] for m in dec.members] == ob.bank_borns()
    deca = DeviceBankDecisions(K=4, retrieve_k=2, mode="a", device=cuda)
    for i in range(6):
        _, R, _ = deca.step(admit=(poses[i], i, i))
    assert R == [0, 1, 2, 3]
    # empty bank retrieval
    dece = DeviceBankDecisions(K=4, retrieve_k=2, device=cuda)
    assert dece.step(target=poses[0])[1] == []


@pytest.mark.parametrize("P", [2, 4, 8])
def test_a2a_pack_unpack_vs_oracle(cuda, P):
    """pack -> (all-to-all of contiguous blocks) -> unpack equals the reference's
    chunk/cat all_to_all for every rank (single GPU holds all ranks' buffers)."""
    from reworld_b200.ulysses import a2a_pack, a2a_unpack
    B, L, H, D = 1, 48, 24, 128
    Ls = L // P
    g = torch.Generator().manual_seed(P)
    shards = [torch.randn(B, Ls, H, D, generator=g).to(torch.bfloat16) for _ in range(P)]
    want = ou.seq_to_head([s.float().numpy() for s in shards])
    packed = [a2a_pack(s.to(cuda), P) for s in shards]             # [P, B, Ls, H/P, D] each
    recv = [torch.stack([packed[src][dst] for src in range(P)]) for dst in range(P)]
    for r in range(P):
        got = recv[r].permute(1, 0, 2, 3, 4).reshape(B, L, H // P, D)   # B = 1: already [L, H/P, D]
        assert np.array_equal(got.float().cpu().numpy(), want[r])
    back_want = ou.head_to_seq(want)
    for r in range(P):
        # rank src holds [L, H/P, D] = recv[src]; its block for rank r is recv[src][r]
        blocks = torch.stack([recv[src][r] for src in range(P)])
        got = a2a_unpack(blocks, H)
        assert np.array_equal(got.float().cpu().numpy(), back_want[r])
    _status_clean()


def test_sp_barrier_single_rank_and_timeout(cuda):
    """rw_sp_barrier completes at once for a group of one, and a wait for a peer
    that never signals ends after its time limit with RW_STATUS_TIMEOUT_PEER in
    the status word (no fault; the context stays usable)."""
    import ctypes
    from reworld_b200 import _native
    lib = _native.lib()
    stream = _native.stream_ptr(cuda)
    sig = torch.zeros(2, 8, dtype=torch.int32, device=cuda)
    ptrs = torch.tensor([sig[0].data_ptr(), sig[1].data_ptr()], dtype=torch.int64, device=cuda)
    st = torch.zeros(4, dtype=torch.int32, device=cuda)
    assert lib.rw_sp_barrier(ctypes.c_void_p(ptrs.data_ptr()), 0, 1, 0, 1, 1000,
                             ctypes.c_void_p(st.data_ptr()), stream) == 0
    torch.cuda.synchronize()
    assert int(st[0]) == 0 and int(sig[0, 0]) == 1
    # two ranks on one device, rank 1 never signals: rank 0's wait runs out after 100 ms
    assert lib.rw_sp_barrier(ctypes.c_void_p(ptrs.data_ptr()), 2, 2, 0, 5, 100,
                             ctypes.c_void_p(st.data_ptr()), stream) == 0
    torch.cuda.synchronize()
    assert int(st[0]) & 0x20
    assert int(sig[0, 2]) == 5 and int(sig[1, 2]) == 5     # rank 0 signalled both arrays
    assert lib.rw_sp_barrier(ctypes.c_void_p(ptrs.data_ptr()), 0, 3, 5, 1, 100, None, stream) == -1   # rank >= P
    x = torch.ones(16, device=cuda)
    assert float((x * 2).sum()) == 32.0                      # context still usable


def test_sp_sync_signal_and_wait_emulated(cuda):
    """The sync record of the peer-memory kernels on one GPU: a scatter of rank 1 of
    4 (owners' buffers and signal arrays local) signals, from its last CTA, epoch 7
    into entry slot + 1 of all four signal arrays and leaves its completion counter
    at zero; rw_sp_wait returns at once for epochs already signalled and, for a
    rank that never signals, ends after its time limit with RW_STATUS_TIMEOUT_PEER
    (no fault; the context stays usable)."""
    import ctypes
    from reworld_b200 import _native
    from reworld_b200._native import RwSpSync, c_vp
    P, rank, H, Ls = 4, 1, 8, 300
    Hp = H // P
    q, k, v = (torch.randn(Ls, H, 128, device=cuda).to(torch.bfloat16) for _ in range(3))
    qd = [torch.zeros(P * Ls, Hp, 128, dtype=torch.bfloat16, device=cuda) for _ in range(P)]
    cd = [torch.zeros(P * Ls, Hp, 128, dtype=torch.bfloat16, device=cuda) for _ in range(2 * P)]
    ptrs = [torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device=cuda) for ts in (qd, cd[:P], cd[P:])]
    sig = torch.zeros(P, 16, dtype=torch.int32, device=cuda)
    sig_ptrs = torch.tensor([sig[p].data_ptr() for p in range(P)], dtype=torch.int64, device=cuda)
    counter = torch.zeros(1, dtype=torch.int32, device=cuda)
    st = torch.zeros(4, dtype=torch.int32, device=cuda)
    lib = _native.lib()
    sync = RwSpSync(c_vp(sig_ptrs.data_ptr()), c_vp(counter.data_ptr()), P, rank, 0, 0, 4, 7, 1000, 0)
    code = lib.rw_sp_scatter_qkv(
        c_vp(q.data_ptr()), c_vp(k.data_ptr()), c_vp(v.data_ptr()), q.stride(0), q.stride(1), k.stride(0),
        k.stride(1), v.stride(0), v.stride(1), *(c_vp(t.data_ptr()) for t in ptrs), Ls, H, 128, P, rank, 0,
        P * Ls, None, ctypes.byref(sync), c_vp(st.data_ptr()), _native.stream_ptr(cuda))
    _native.check(code, "rw_sp_scatter_qkv")
    torch.cuda.synchronize()
    assert all(int(sig[p, 4 + rank]) == 7 for p in range(P)) and int(sig[:, 4:8].sum()) == 7 * P
    assert int(counter[0]) == 0 and int(st[0]) == 0
    assert torch.equal(qd[2][rank * Ls:(rank + 1) * Ls], q[:, 2 * Hp:3 * Hp])
    # a wait on entries 4..7 of rank 0's array: only entry 5 (rank 1) holds an epoch
    sig[0, 4:8] = 7
    w_ok = RwSpSync(c_vp(sig_ptrs.data_ptr()), None, P, 0, 4, 7, 0, 0, 1000, 0)
    assert lib.rw_sp_wait(ctypes.byref(w_ok), c_vp(st.data_ptr()), _native.stream_ptr(cuda)) == 0
    torch.cuda.synchronize()
    assert int(st[0]) == 0
    w_late = RwSpSync(c_vp(sig_ptrs.data_ptr()), None, P, 2, 4, 8, 0, 0, 100, 0)   # nobody signals epoch 8
    assert lib.rw_sp_wait(ctypes.byref(w_late), c_vp(st.data_ptr()), _native.stream_ptr(cuda)) == 0
    torch.cuda.synchronize()
    assert int(st[0]) & 0x20
    assert lib.rw_sp_wait(None, None, _native.stream_ptr(cuda)) == -1
    x = torch.ones(16, device=cuda)
    assert float((x * 2).sum()) == 32.0


@pytest.mark.parametrize("P,rank", [(1, 0), (2, 1), (4, 2)])
def test_sp_scatter_qkv_emulated_ranks(cuda, P, rank):
    """rw_sp_scatter_qkv of rank `rank` of P on one GPU: the P owners' buffers are
    local tensors (the kernel only stores through its pointer arrays and waits on
    nothing).  q rows, v cache rows and RoPE(+PM-RoPE) k cache rows land at the
    owner's local head, bit-exact against the oracle."""
    from reworld_b200 import RopeArgs, _native, device_table
    from reworld_b200._native import c_vp
    f, h, w = 3, 4, 5
    ct = f * h * w + 4                       # 4 tokens past the grid stay unroped
    H, Ls = 8, ct // P
    Hp = H // P
    gen = torch.Generator().manual_seed(70 + P)
    q, k, v = ((torch.randn(Ls, H, 128, generator=gen) * 2).to(torch.bfloat16) for _ in range(3))
    delta = torch.randn(1, f, 64, generator=gen) * 0.4
    freqs = orope.build_freqs(128, gi.ROPE_SCALE_H, gi.ROPE_SCALE_W)
    cap, d0 = 2 * ct, 10
    qd = [torch.zeros(P * Ls, Hp, 128, dtype=torch.bfloat16, device=cuda) for _ in range(P)]
    ckd = [torch.zeros(cap, Hp, 128, dtype=torch.bfloat16, device=cuda) for _ in range(P)]
    cvd = [torch.zeros(cap, Hp, 128, dtype=torch.bfloat16, device=cuda) for _ in range(P)]
    ptrs = [torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device=cuda) for ts in (qd, ckd, cvd)]
    rope = RopeArgs(device_table(freqs, cuda), (f, h, w), 9, delta=delta.to(cuda))
    rs = rope.struct()
    qg, kg, vg = q.to(cuda), k.to(cuda), v.to(cuda)
    code = _native.lib().rw_sp_scatter_qkv(
        c_vp(qg.data_ptr()), c_vp(kg.data_ptr()), c_vp(vg.data_ptr()), qg.stride(0), qg.stride(1),
        kg.stride(0), kg.stride(1), vg.stride(0), vg.stride(1), *(c_vp(t.data_ptr()) for t in ptrs),
        Ls, H, 128, P, rank, d0, cap, ctypes.byref(rs), None, None, _native.stream_ptr(cuda))
    _native.check(code, "rw_sp_scatter_qkv")
    torch.cuda.synchronize()
    # the oracle's roped k for this rank's tokens (chunk positions rank * Ls + s)
    kfull = torch.zeros(1, ct, H, 128, dtype=torch.bfloat16)
    kfull[0, rank * Ls:(rank + 1) * Ls] = k
    kr = orope.causal_rope_apply(kfull.float().numpy(), [(f, h, w)], freqs, start_frame=9)
    cs = rope.delta_cs.cpu()                                                   # [1, f, 64, 2]
    tok = cs.unsqueeze(2).expand(-1, -1, h * w, -1, -1).reshape(1, f * h * w, 1, 64, 2)
    tok = torch.cat([tok, torch.zeros(1, ct - f * h * w, 1, 64, 2)], dim=1).numpy()
    kr = orope.pm_rope_apply_cs(kr, tok[..., 0], tok[..., 1])
    kr[:, f * h * w:] = kfull.float().numpy()[:, f * h * w:]
    want_k = f32_to_bf16_bits(kr)[0, rank * Ls:(rank + 1) * Ls]              # [Ls, H, 128]
    t0, t1 = rank * Ls, (rank + 1) * Ls
    for p in range(P):
        hs = slice(p * Hp, (p + 1) * Hp)
        assert torch.equal(qd[p][t0:t1].cpu(), q[:, hs])
        assert torch.equal(cvd[p][d0 + t0:d0 + t1].cpu(), v[:, hs])
        assert np.array_equal(torch_bf16_to_bits(ckd[p][d0 + t0:d0 + t1]), want_k[:, hs])
        assert not qd[p][:t0].any() and not qd[p][t1:].any()
        assert not ckd[p][:d0 + t0].any() and not ckd[p][d0 + t1:].any()


def test_rope_store_two_batches_with_q_and_phase(cuda):
    """B = 2 with a per-batch PM-RoPE phase and the optional roped q copy: every
    row bit-exact against the oracle (the kernel walks tokens of both batches)."""
    from reworld_b200 import RopeArgs, device_table, rope_kv_store
    gen = torch.Generator().manual_seed(81)
    f, h, w, H = 3, 4, 5, 3
    B, L = 2, f * h * w + 4
    k, v, q = ((torch.randn(B, L, H, 128, generator=gen) * 2).to(torch.bfloat16) for _ in range(3))
    delta = torch.randn(B, f, 64, generator=gen) * 0.4
    freqs = orope.build_freqs(128, gi.ROPE_SCALE_H, gi.ROPE_SCALE_W)
    ck = torch.zeros(B, L + 9, H, 128, dtype=torch.bfloat16, device=cuda)
    cv = torch.zeros_like(ck)
    rope = RopeArgs(device_table(freqs, cuda), (f, h, w), 5, delta=delta.to(cuda))
    q_out = rope_kv_store(k.to(cuda), v.to(cuda), ck, cv, 9, rope=rope, q=q.to(cuda))
    torch.cuda.synchronize()
    cs = rope.delta_cs.cpu()
    tok = cs.unsqueeze(2).expand(-1, -1, h * w, -1, -1).reshape(B, f * h * w, 1, 64, 2)
    tok = torch.cat([tok, torch.zeros(B, L - f * h * w, 1, 64, 2)], dim=1).numpy()

    def want(x):
        y = orope.causal_rope_apply(x.float().numpy(), [(f, h, w)] * B, freqs, start_frame=5)
        y = orope.pm_rope_apply_cs(y, tok[..., 0], tok[..., 1])
        y[:, f * h * w:] = x.float().numpy()[:, f * h * w:]
        return f32_to_bf16_bits(y)

    assert np.array_equal(torch_bf16_to_bits(ck[:, 9:]), want(k))
    assert np.array_equal(torch_bf16_to_bits(q_out), want(q))
    assert torch.equal(cv[:, 9:].cpu(), v) and not ck[:, :9].any() and not cv[:, :9].any()
