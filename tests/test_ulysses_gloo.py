"""Ulysses exchange logic on CPU: world_size 2 and 4 gloo process groups run the
package's block exchange (exchange_blocks / blocks_to_seq / seq_to_blocks, one
all_to_all_single per direction) with the pack/unpack layouts restated here on
the CPU (the CUDA pack/unpack kernels are checked against the same layouts in
tests/test_gpu_kernels.py), and must reproduce the reference's
wan_5b/distributed/util.py:52-64 all_to_all results (tests/golden/ulysses.npz)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _pack(x, P):
    """[B, Ls, H, D] -> [P, B, Ls, H/P, D], block p = head group p."""
    B, Ls, H, D = x.shape
    return x.reshape(B, Ls, P, H // P, D).permute(2, 0, 1, 3, 4).contiguous()


def _unpack(blocks):
    """[P, B, Ls, H/P, D] -> [B, Ls, H, D]."""
    P, B, Ls, Hp, D = blocks.shape
    return blocks.permute(1, 2, 0, 3, 4).reshape(B, Ls, P * Hp, D)


def _worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import torch.distributed as dist
    import inputs as gi
    from reworld_b200.ulysses import blocks_to_seq, exchange_blocks, seq_to_blocks
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    x = gi.ulysses_shard(rank, world)                                  # [1, L/P, H, D]
    y = blocks_to_seq(exchange_blocks(_pack(x, world)))                # seq -> head
    z = _unpack(exchange_blocks(seq_to_blocks(y, world)))              # head -> seq
    np.savez(os.path.join(out_dir, f"r{rank}.npz"), y=y.numpy(), z=z.numpy())
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_exchange_matches_reference_all_to_all(tmp_path, world):
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    g = np.load(os.path.join(ROOT, "tests", "golden", "ulysses.npz"))
    for r in range(world):
        d = np.load(tmp_path / f"r{r}.npz")
        np.testing.assert_array_equal(d["y"], g[f"p{world}_r{r}_y"])
        np.testing.assert_array_equal(d["z"], g[f"p{world}_r{r}_z"])
