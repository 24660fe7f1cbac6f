"""Tensor-parallel forward on 2 GPUs (skipped with fewer): each rank holds
the same seeded model, shards it by rows (peer-store gathers over the
communicator), and must (1) return the unsharded model's logits: bit for
bit for the K-quant model with BREW_TP_EXACT=1 (K split as on one GPU; the
gathers copy), within 1e-6 relative L2 with the default per-shard K split
(the Q8_0 model runs the persistent decode kernel unsharded, another
summation order, and is checked against the oracle only); (2) match the
oracle's logits within 1e-4 relative L2 and its greedy tokens exactly.
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rel(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b.astype(np.float64)))


def _configs():
    from brewference_b200 import config as C
    kq = C.qwen25_7b().replace(dim=1024, hidden_dim=2048, n_heads=8, n_kv_heads=4, n_layers=3, vocab_size=4096,
                               seq_len=128)
    q8 = C.qwen3_1_7b().replace(n_layers=2, vocab_size=4096, seq_len=128)
    # (name, config, BREW_TP_EXACT, against the unsharded model: "exact", "close" or None)
    return [("qwen2-kquant-exact", kq, True, "exact"), ("qwen2-kquant", kq, False, "close"),
            ("qwen3-q8_0", q8, False, None)]


def _rank(rank, port, results):
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=120))
    comm = None
    try:
        import oracle
        from brewference_b200 import _native as N
        from brewference_b200.api import Communicator, DeviceModel, comm_unique_id
        N.init(rank)
        box = [comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        comm = Communicator(box[0], WORLD, rank)
        out = {}
        for name, cfg, exact_env, vs_one in _configs():
            seed = 17
            dm = DeviceModel.synthesize(cfg, seed)
            if exact_env:
                os.environ["BREW_TP_EXACT"] = "1"
            else:
                os.environ.pop("BREW_TP_EXACT", None)
            dm.set_tp(comm)
            prompt = np.random.default_rng(seed).integers(0, cfg.vocab_size, 8).tolist()
            dm.reset()
            lg_tp = [dm.forward([prompt[i]], [i])[0][0].copy() for i in range(3)]
            toks_tp = dm.generate(prompt, 24)
            dm.close()
            ref = DeviceModel.synthesize(cfg, seed)   # unsharded, this GPU
            ref.reset()
            lg_1 = [ref.forward([prompt[i]], [i])[0][0].copy() for i in range(3)]
            ref.close()
            om = oracle.OracleModel(cfg, seed)
            om.reset()
            lg_o = [om.forward(prompt[i], i) for i in range(3)]
            toks_o = om.generate(prompt, 24)
            om.close()
            for i in range(3):
                assert _rel(lg_tp[i], lg_o[i]) < 1e-4, (name, i, _rel(lg_tp[i], lg_o[i]))
                if vs_one == "exact":
                    assert np.array_equal(lg_tp[i], lg_1[i]), (name, i)
                elif vs_one == "close":
                    assert _rel(lg_tp[i], lg_1[i]) < 1e-6, (name, i, _rel(lg_tp[i], lg_1[i]))
            assert toks_tp == toks_o, (name, toks_tp, toks_o)
            out[name] = "ok"
        results[rank] = out
    except Exception as e:   # noqa: BLE001 - reported to the parent
        results[rank] = repr(e)
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_tp_two_gpus():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank, args=(r, port, results)) for r in range(WORLD)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=600)
        got = dict(results)
    want = {name: "ok" for name, _, _, _ in _configs()}
    assert got == {0: want, 1: want}, got
