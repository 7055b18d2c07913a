"""The column split and the head split on two GPUs (skipped with fewer).

Column split: two ranks (NCCL) each own one of the tiny checkpoint's two sequences and half
of its FFN and vocabulary columns; greedy ``generate_batch_ids`` on each rank must
reproduce the tokens the reference's own ``orchard/model.py`` produced for that sequence
(tests/golden/tiny_model.npz), with the decode step captured in CUDA graphs and eagerly.
The prompts have different lengths, so the shorter rank's prefill is padded into the
scratch slot. Head split: both ranks run both sequences, each with half of the heads."""

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "tiny_model.npz")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, graphs, q, heads=False):
    import datetime
    import json

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    llm = None
    try:
        from orchard_b200.model import Llama
        z = np.load(GOLDEN)
        cfg = json.loads(str(z["config_json"]))
        ckpt = {k[len("ckpt/"):]: z[k] for k in z.files if k.startswith("ckpt/")}
        prompts = [[int(v) for v in p if v >= 0] for p in z["prompts"]]
        llm = Llama.from_tensors(cfg, ckpt, device=rank, max_batch=2, use_graphs=graphs, group=dist.group.WORLD,
                                 split_heads=heads)
        if heads:  # every rank runs both sequences with one of the two heads
            toks = llm.generate_batch_ids(prompts, max_tokens=int(z["max_tokens"]), temperature=0)
            q.put((rank, toks, None))
        else:
            toks = llm.generate_batch_ids([prompts[rank]], max_tokens=int(z["max_tokens"]), temperature=0)
            q.put((rank, toks[0], None))
    except Exception as e:  # reported to the parent
        q.put((rank, None, repr(e)))
    finally:
        if llm is not None:
            llm.engine.release_graphs()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("graphs", [True, False])
def test_column_split_two_gpus_matches_reference_golden(graphs):
    import torch.multiprocessing as mp
    z = np.load(GOLDEN)
    ref = [[int(v) for v in t if v >= 0] for t in z["tokens"]]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, graphs, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        r, t, err = q.get(timeout=300)
        assert err is None, err
        got[r] = t
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert [got[0], got[1]] == ref


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("graphs", [True, False])
def test_head_split_two_gpus_matches_reference_golden(graphs):
    """The head split: both ranks run both sequences, each holding one of the tiny model's two
    attention heads (its Q/K/V rows, O columns and KV cache) and half of the FFN and
    vocabulary; both must produce the reference's golden tokens for both sequences."""
    import torch.multiprocessing as mp
    z = np.load(GOLDEN)
    ref = [[int(v) for v in t if v >= 0] for t in z["tokens"]]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, graphs, q, True)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        r, t, err = q.get(timeout=300)
        assert err is None, err
        got[r] = t
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert got[0] == ref and got[1] == ref


def _ar_rank(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from orchard_b200._lib import call
        from orchard_b200.model import _PeerAllReduce
        call("orch_init", rank, None)
        H, rows_max = 4096, 64
        ar = _PeerAllReduce(dist.group.WORLD, world, rank, rows_max * H, dev)
        ok = [ar.ok]
        for it, rows in enumerate([1, 64, 3, 8, 64, 2, 37]):  # 8..296 blocks, both banks
            g = torch.Generator(device=dev).manual_seed(1000 * it + rank)
            x = torch.randn((rows_max, H), generator=g, device=dev)
            parts = [torch.empty((rows, H), device=dev) for _ in range(world)]
            dist.all_gather(parts, x[:rows].contiguous())
            want = parts[0].clone()
            for p in parts[1:]:
                want += p  # rank order, fp32: the kernel's order
            tail = x[rows:].clone()
            ar(x, rows * H, algo=1 + it % 2)  # one shot and two shots in turn
            torch.cuda.synchronize(dev)
            ok.append(bool(torch.equal(x[:rows], want)) and bool(torch.equal(x[rows:], tail)))
        import ctypes as C
        flags = C.c_uint32(0)
        call("orch_device_check", C.byref(flags), torch.cuda.current_stream(dev).cuda_stream)
        q.put((rank, ok, flags.value, None))
    except Exception as e:
        q.put((rank, None, None, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_allreduce_two_gpus_bit_exact():
    """orch_peer_allreduce over two GPUs equals the rank-ordered fp32 sum of the gathered
    inputs, bit for bit, on every rank, over calls of 1..64 rows (both banks of slots), with
    the one-shot and the two-shot form in turn."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ar_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for _ in range(2):
        r, ok, flags, err = q.get(timeout=300)
        assert err is None, err
        assert all(ok), ok
        assert flags == 0
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
