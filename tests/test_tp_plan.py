"""Host logic of the tensor-parallel forward on CPU: two gloo ranks split
matrices by rows with brew_tp_rows (the C ABI's plan, no GPU needed), each
multiplies its rows with the oracle, and the all-gathered slices in rank
order must equal the unsharded product exactly (a row's arithmetic does not
depend on the split).  The sharded argmax (per-rank (value, index) keys,
maximum over ranks, first index on ties) must equal the global argmax.
"""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from brewference_b200 import _native as N
from brewference_b200 import config as C
from brewference_b200.api import tp_rows


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _key(v, idx):
    u = np.float32(v).view(np.uint32).item()
    u = (~u & 0xFFFFFFFF) if (u & 0x80000000) else (u | 0x80000000)
    return (u << 32) | (0xFFFFFFFF - idx)


def _rank(rank, world, port, results):
    import torch
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        for qt, K, Nr in [(C.TYPE_Q8_0, 256, 96), (C.TYPE_Q4_0, 512, 64), (C.TYPE_Q4_K, 512, 32),
                          (C.TYPE_Q6_K, 256, 48)]:
            w = oracle.synth_quantized(qt, 31, 4, Nr * K)
            x = oracle.synth_fill(31, 5, 0, K, 1.0)
            r0, r1 = tp_rows(Nr, world, rank)
            part = oracle.matvec(qt, w, r0 * K, x, K, r1 - r0)
            parts = [torch.zeros(Nr // world, dtype=torch.float32) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(part))
            full = np.concatenate([p.numpy() for p in parts])
            want = oracle.matvec(qt, w, 0, x, K, Nr)
            assert np.array_equal(full, want), (qt, rank)
            # sharded argmax with ties: force the maximum into both halves
            lg = want.copy()
            lg[1] = lg[Nr // world + 1] = lg.max() + 1.0
            mine = lg[r0:r1]
            i = int(np.argmax(mine))
            keys = [None] * world
            dist.all_gather_object(keys, _key(mine[i], r0 + i))
            best = max(keys)
            assert 0xFFFFFFFF - (best & 0xFFFFFFFF) == int(np.argmax(lg)) == 1
        results[rank] = "ok"
    except Exception as e:   # noqa: BLE001 - reported to the parent
        results[rank] = repr(e)
    finally:
        dist.destroy_process_group()


def test_row_split_gather_equals_full():
    world = 2
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank, args=(r, world, port, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
        assert dict(results) == {0: "ok", 1: "ok"}, dict(results)



def test_tp_rows_plan_and_errors():
    assert tp_rows(3584, 8, 0) == (0, 448)
    assert tp_rows(3584, 8, 7) == (3136, 3584)
    assert tp_rows(152064, 4, 3) == (114048, 152064)
    with pytest.raises(N.BrewError):
        tp_rows(1000, 3, 0)            # rows must split evenly
    with pytest.raises(N.IllegalArgumentException):
        tp_rows(1024, 2, 2)            # rank out of range
