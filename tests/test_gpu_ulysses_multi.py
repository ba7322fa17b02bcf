"""Ulysses head-parallel chunk attention on 2 GPUs (one process per GPU, NCCL)
against the single-GPU result on the same inputs: max-abs 2e-2, mean-abs 2e-3
(only the floating-point summation order differs).  Skipped with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
F, HT, WT, H = 3, 11, 20, 8            # 660-token chunk, 8 heads
L = F * HT * WT
N_CACHED = 3


def _inputs():
    g = torch.Generator().manual_seed(77)
    q = torch.randn(1, L, H, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(1, L, H, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(1, L, H, 128, generator=g).to(torch.bfloat16)
    ck = torch.randn(1, (N_CACHED + 1) * L, H, 128, generator=g).to(torch.bfloat16)
    cv = torch.randn(1, (N_CACHED + 1) * L, H, 128, generator=g).to(torch.bfloat16)
    return q, k, v, ck, cv


def _worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    import datetime
    import torch.distributed as dist
    from reworld_b200 import RopeArgs, build_freqs, device_table
    from reworld_b200.ulysses import sp_chunk_attention
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    q, k, v, ck, cv = _inputs()
    Ls, Hp = L // world, H // world
    sl = slice(rank * Ls, (rank + 1) * Ls)
    hs = slice(rank * Hp, (rank + 1) * Hp)
    rope = RopeArgs(device_table(build_freqs(128, 12 / 22, 20 / 40), dev), (F, HT, WT), N_CACHED * F)
    out = sp_chunk_attention(q[:, sl].to(dev), k[:, sl].to(dev), v[:, sl].to(dev),
                             ck[:, :, hs].contiguous().to(dev), cv[:, :, hs].contiguous().to(dev),
                             N_CACHED * L, rope=rope)
    torch.cuda.synchronize()
    np.save(os.path.join(out_dir, f"r{rank}.npy"), out.float().cpu().numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_ulysses_two_gpus_match_single_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from reworld_b200 import RopeArgs, build_freqs, chunk_attention, device_table, rope_kv_store
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.spawn(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    dev = torch.device("cuda", 0)
    q, k, v, ck, cv = _inputs()
    ck, cv = ck.to(dev), cv.to(dev)
    rope = RopeArgs(device_table(build_freqs(128, 12 / 22, 20 / 40), dev), (F, HT, WT), N_CACHED * F)
    rope_kv_store(k.to(dev), v.to(dev), ck, cv, N_CACHED * L, rope=rope)
    ref = chunk_attention(q.to(dev), ck, cv, rope=rope).float().cpu().numpy()
    got = np.concatenate([np.load(tmp_path / f"r{r}.npy") for r in range(2)], axis=1)
    err = np.abs(got - ref)
    assert err.max() < 2e-2 and err.mean() < 2e-3, (err.max(), err.mean())


def _p2p_worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    import datetime
    import torch.distributed as dist
    from reworld_b200 import RopeArgs, build_freqs, device_table, _native
    from reworld_b200.ulysses import UlyssesP2P
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    q, k, v, ck, cv = _inputs()
    Ls, Hp = L // world, H // world
    sl = slice(rank * Ls, (rank + 1) * Ls)
    hs = slice(rank * Hp, (rank + 1) * Hp)
    sp = UlyssesP2P(dist.group.WORLD, 1, (N_CACHED + 1) * L, L, H, device=dev)
    n0 = N_CACHED * L
    sp.cache_k(0)[:, :n0].copy_(ck[:, :n0, hs].to(dev))
    sp.cache_v(0)[:, :n0].copy_(cv[:, :n0, hs].to(dev))
    rope = RopeArgs(device_table(build_freqs(128, 12 / 22, 20 / 40), dev), (F, HT, WT), N_CACHED * F)
    outs = []
    for rep in range(2):                         # twice: buffers are reused across calls
        out = sp.layer(0, q[:, sl].to(dev), k[:, sl].to(dev), v[:, sl].to(dev), n0, rope=rope)
        outs.append(out.float().cpu().numpy())
    torch.cuda.synchronize()
    _native.check_status(dev)
    np.save(os.path.join(out_dir, f"p2p_r{rank}.npy"), outs[-1])
    np.save(os.path.join(out_dir, f"p2p_first_r{rank}.npy"), outs[0])
    np.save(os.path.join(out_dir, f"p2p_k_r{rank}.npy"), sp.cache_k(0)[:, n0:n0 + L].float().cpu().numpy())
    dist.barrier()
    del sp
    dist.destroy_process_group()


def test_ulysses_p2p_two_gpus_match_single_gpu(tmp_path):
    """Peer-memory exchanges (RoPE + cache write fused into the seq->head scatter)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from reworld_b200 import RopeArgs, build_freqs, chunk_attention, device_table, rope_kv_store
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.spawn(_p2p_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    dev = torch.device("cuda", 0)
    q, k, v, ck, cv = _inputs()
    ck, cv = ck.to(dev), cv.to(dev)
    rope = RopeArgs(device_table(build_freqs(128, 12 / 22, 20 / 40), dev), (F, HT, WT), N_CACHED * F)
    n0 = N_CACHED * L
    rope_kv_store(k.to(dev), v.to(dev), ck, cv, n0, rope=rope)
    ref = chunk_attention(q.to(dev), ck, cv, rope=rope).float().cpu().numpy()
    got = np.concatenate([np.load(tmp_path / f"p2p_r{r}.npy") for r in range(2)], axis=1)
    first = np.concatenate([np.load(tmp_path / f"p2p_first_r{r}.npy") for r in range(2)], axis=1)
    for g in (got, first):
        err = np.abs(g - ref)
        assert err.max() < 2e-2 and err.mean() < 2e-3, (err.max(), err.mean())
    # the owning ranks' caches hold the same roped K rows as the single-GPU cache (bit for bit)
    kr = ck[:, n0:n0 + L].float().cpu().numpy()
    Hp = H // 2
    for r in range(2):
        np.testing.assert_array_equal(np.load(tmp_path / f"p2p_k_r{r}.npy"), kr[:, :, r * Hp:(r + 1) * Hp])


def _single_rank_worker(rank, world, port, out_dir):
    """A group of one: the scatter signals its own rank, the attention waits for it
    and signals again; five layer() calls alternate the q / output copies, with and
    without the output wait."""
    import sys
    sys.path.insert(0, ROOT)
    import datetime
    import torch.distributed as dist
    from reworld_b200 import RopeArgs, build_freqs, device_table, _native
    from reworld_b200.ulysses import UlyssesP2P
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=120), device_id=dev)
    q, k, v, ck, cv = _inputs()
    sp = UlyssesP2P(dist.group.WORLD, 2, (N_CACHED + 1) * L, L, H, device=dev)
    n0 = N_CACHED * L
    for layer in range(2):
        sp.cache_k(layer)[:, :n0].copy_(ck[:, :n0].to(dev))
        sp.cache_v(layer)[:, :n0].copy_(cv[:, :n0].to(dev))
    rope = RopeArgs(device_table(build_freqs(128, 12 / 22, 20 / 40), dev), (F, HT, WT), N_CACHED * F)
    outs = []
    for call in range(5):
        out = sp.layer(call % 2, q.to(dev), k.to(dev), v.to(dev), n0, rope=rope, sync_output=call % 2 == 0)
        if call % 2 == 1:
            sp.finish()
        outs.append(out.float().cpu().numpy())
    torch.cuda.synchronize()
    _native.check_status(dev)
    np.save(os.path.join(out_dir, "single.npy"), np.stack(outs))
    np.save(os.path.join(out_dir, "single_counters.npy"), sp.counters.cpu().numpy())
    dist.barrier()
    del sp
    dist.destroy_process_group()


def test_ulysses_p2p_group_of_one_matches_chunk_attention(cuda, tmp_path):
    """UlyssesP2P with one rank on one GPU (the scatter's signal and the attention's
    wait and signal all on this rank, in stream order): every call equals the
    single-GPU attention, and the completion counters end at zero."""
    from reworld_b200 import RopeArgs, build_freqs, chunk_attention, device_table, rope_kv_store
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.spawn(_single_rank_worker, args=(1, port, str(tmp_path)), nprocs=1, join=True)
    q, k, v, ck, cv = _inputs()
    ck, cv = ck.to(cuda), cv.to(cuda)
    rope = RopeArgs(device_table(build_freqs(128, 12 / 22, 20 / 40), cuda), (F, HT, WT), N_CACHED * F)
    n0 = N_CACHED * L
    rope_kv_store(k.to(cuda), v.to(cuda), ck, cv, n0, rope=rope)
    ref = chunk_attention(q.to(cuda), ck, cv, rope=rope).float().cpu().numpy()
    got = np.load(tmp_path / "single.npy")
    for g in got:
        err = np.abs(g - ref)
        assert err.max() < 2e-2 and err.mean() < 2e-3, (err.max(), err.mean())
    assert not np.load(tmp_path / "single_counters.npy").any()


def _seq_kv_worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    import datetime
    import torch.distributed as dist
    from reworld_b200 import RopeArgs, build_freqs, device_table
    from reworld_b200.ulysses import sp_chunk_attention_seq_kv
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    q, k, v, ck, cv = _inputs()
    Ls = L // world
    n0 = N_CACHED * L
    sl = slice(rank * Ls, (rank + 1) * Ls)
    cs = slice(rank * (n0 // world), (rank + 1) * (n0 // world))   # this rank's cached keys, all heads
    rope = RopeArgs(device_table(build_freqs(128, 12 / 22, 20 / 40), dev), (F, HT, WT), N_CACHED * F)
    work = tuple(torch.empty((1, n0 + L + 16, H // world, 128), dtype=torch.bfloat16, device=dev) for _ in range(2))
    outs = []
    for rep in range(2):                         # twice: the work buffers are reused
        out = sp_chunk_attention_seq_kv(q[:, sl].to(dev), k[:, sl].to(dev), v[:, sl].to(dev),
                                        ck[:, cs].contiguous().to(dev), cv[:, cs].contiguous().to(dev),
                                        rope=rope, work=work if rep else None)
        outs.append(out.float().cpu().numpy())
    torch.cuda.synchronize()
    np.save(os.path.join(out_dir, f"seqkv_r{rank}.npy"), outs[-1])
    np.save(os.path.join(out_dir, f"seqkv_first_r{rank}.npy"), outs[0])
    dist.barrier()
    dist.destroy_process_group()


def test_ulysses_sequence_sharded_cache_two_gpus_match_single_gpu(tmp_path):
    """The cache sharded along the sequence (every rank a slice of the cached keys,
    all heads), moved seq -> head with the chunk's q/k/v in every call."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from reworld_b200 import RopeArgs, build_freqs, chunk_attention, device_table, rope_kv_store
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.spawn(_seq_kv_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    dev = torch.device("cuda", 0)
    q, k, v, ck, cv = _inputs()
    ck, cv = ck.to(dev), cv.to(dev)
    rope = RopeArgs(device_table(build_freqs(128, 12 / 22, 20 / 40), dev), (F, HT, WT), N_CACHED * F)
    rope_kv_store(k.to(dev), v.to(dev), ck, cv, N_CACHED * L, rope=rope)
    ref = chunk_attention(q.to(dev), ck, cv, rope=rope).float().cpu().numpy()
    for name in ("seqkv_first_r", "seqkv_r"):
        got = np.concatenate([np.load(tmp_path / f"{name}{r}.npy") for r in range(2)], axis=1)
        err = np.abs(got - ref)
        assert err.max() < 2e-2 and err.mean() < 2e-3, (name, err.max(), err.mean())
