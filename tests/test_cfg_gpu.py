"""CFG-parallel combine (cfg_parallel.py:48-71) on the GPU against the CPU restatement: bit-exact."""

import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import cfg as ocfg

pytestmark = pytest.mark.gpu


def _branches(shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g).to(dtype), (torch.randn(shape, generator=g) * 0.7).to(dtype))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(1, 16, 21, 60, 104), (1, 16, 3, 12, 20), (1001,), (7,)])
@pytest.mark.parametrize("scale", [5.0, 3.5])
def test_cfg_combine_bit_exact(pkg, dev, dtype, shape, scale):
    pos, neg = _branches(shape, dtype, 3)
    got = pkg.cfg_combine(pos.to(dev), neg.to(dev), scale).cpu()
    ref = ocfg.cfg_combine_ref(pos.float().numpy(), neg.float().numpy(), scale, dtype == torch.bfloat16)
    assert np.array_equal(got.float().numpy().view(np.uint32), ref.view(np.uint32))


def test_cfg_combine_in_place_and_errors(pkg, dev):
    pos, neg = _branches((4099,), torch.bfloat16, 4)
    ref = ocfg.cfg_combine_ref(pos.float().numpy(), neg.float().numpy(), 4.0, True)
    p = pos.to(dev)
    out = pkg.cfg_combine(p, neg.to(dev), 4.0, out=p)
    assert out.data_ptr() == p.data_ptr()
    assert np.array_equal(p.cpu().float().numpy().view(np.uint32), ref.view(np.uint32))
    with pytest.raises(ValueError):
        pkg.cfg_combine(p, neg.to(dev)[:10], 4.0)
    with pytest.raises(TypeError):
        pkg.cfg_combine(p.half(), neg.to(dev).half(), 4.0)
    with pytest.raises(RuntimeError):
        pkg.cfg_combine(pos, neg, 4.0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, out_q):
    try:
        from datetime import timedelta
        from importlib import import_module

        import torch.distributed as dist

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=2, timeout=timedelta(seconds=60), device_id=dev)
        pkg = import_module("vllm-omni-neuron_b200")
        try:
            preds = [_branches((1, 16, 21, 60, 104), torch.bfloat16, 10)[0], _branches((1, 16, 21, 60, 104), torch.bfloat16, 11)[0]]
            out = pkg.cfg_gather_combine(preds[rank].to(dev), 5.0).cpu()
            ref = ocfg.cfg_gather_combine_ref([p.float().numpy() for p in preds], 5.0, True)
            same = bool(np.array_equal(out.float().numpy().view(np.uint32), ref.view(np.uint32)))
            out_q.put((rank, same, None))
        finally:
            dist.destroy_process_group()
    except Exception:
        out_q.put((rank, False, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs >= 2 GPUs")
def test_cfg_gather_combine_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, same, tb in res:
        assert tb is None, tb
        assert same, f"rank {rank}: combine differs from the oracle"
