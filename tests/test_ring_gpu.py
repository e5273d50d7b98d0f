"""Multi-GPU ring attention (one process per GPU, NCCL) against the CPU oracle.
Skips unless at least two CUDA devices are visible."""

import math
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard(rank, b, s, h, seed=21):
    g = torch.Generator().manual_seed(seed + rank)
    return [(torch.randn(b, s, h, 128, generator=g) * 0.6).to(torch.bfloat16) for _ in range(3)]


def _worker(rank, world, port, shapes, out_q):
    try:
        from datetime import timedelta
        from importlib import import_module

        import torch.distributed as dist

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        pkg = import_module("vllm-omni-neuron_b200")
        lib = import_module("vllm-omni-neuron_b200._lib")
        from oracle import attention as oat

        errs = []
        for (b, s, h) in shapes:
            shards = [_shard(r, b, s, h) for r in range(world)]
            q, k, v = (x.to(dev) for x in shards[rank])
            for call in range(2):  # two calls: exercises both send-buffer parities
                o, lse = pkg.ring_attention_const_max_fwd(q, k, v, num_workers=world, training=True)
                od = pkg.wan_cp_self_attention(q, k, v, 1 / math.sqrt(128), world, dist.group.WORLD, None)
            torch.cuda.synchronize()
            # pinned host shards: head groups streamed through the ring, bit-identical to the device call
            oh = pkg.wan_cp_self_attention(*(x.pin_memory() for x in shards[rank]), 1 / math.sqrt(128), world,
                                           dist.group.WORLD, None)
            errs.append(("host_equal", (b, s, h), float(oh.device.type == "cpu" and torch.equal(oh, od.cpu()))))
            f = lambda t: t.float().cpu().numpy()
            qs, ks, vs = ([f(sh[i]) for sh in shards] for i in range(3))
            ref_o, ref_l = oat.const_max_ring_attention(qs, ks, vs, training=True)
            exact = oat.wan_cp_self_attention_oracle(qs, ks, vs, 1 / math.sqrt(128))[rank]
            got = f(o).astype(np.float64)
            r = ref_o[rank].astype(np.float64)
            cos = (got * r).sum() / math.sqrt((got * got).sum() * (r * r).sum())
            errs.append(("cos_ring", (b, s, h), float(cos)))
            errs.append(("max_ring", (b, s, h), float(np.abs(got - r).max())))
            errs.append(("max_exact_dmajor", (b, s, h), float(np.abs(f(od) - exact).max())))
            errs.append(("max_lse", (b, s, h), float(np.abs(f(lse) - ref_l[rank]).max())))
        status = lib.device_status()
        pkg.destroy_rings()
        dist.destroy_process_group()
        out_q.put((rank, errs, status, None))
    except Exception:
        out_q.put((rank, None, None, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs >= 2 GPUs")
def test_ring_multi_gpu():
    world = min(torch.cuda.device_count(), 4)
    shapes = [(1, 256, 2), (1, 200, 3), (2, 130, 1)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, shapes, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for rank, errs, status, tb in res:
        assert tb is None, tb
        assert status == 0
        for name, shape, val in errs:
            if name == "host_equal":
                assert val == 1.0, (rank, name, shape)
            elif name.startswith("cos"):
                assert val >= 0.9999, (rank, name, shape, val)
            elif name == "max_lse":
                assert val <= 3e-2, (rank, name, shape, val)
            else:
                assert val <= 2e-2, (rank, name, shape, val)


def _block_worker(rank, world, port, out_q):
    """CFGP=2 x CP=world/2 transformer block: each rank's shard of the ring result must match the
    same branch computed at CP=1 on one GPU."""
    try:
        import sys
        from datetime import timedelta
        from importlib import import_module

        import torch.distributed as dist

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        pkg = import_module("vllm-omni-neuron_b200")
        rope = import_module("vllm-omni-neuron_b200.rope")
        sys.path.insert(0, os.path.dirname(__file__))
        from test_block_gpu import make_block

        cp = world // 2
        branch, cp_rank = rank // cp, rank % cp
        groups = tuple(tuple(range(g * cp, (g + 1) * cp)) for g in range(2))
        H, heads = 256, 2
        w, hidden, temb, ctx, cos, sin = make_block(1, (3, 16, 16), H, 512, 40, seed=branch)
        S = hidden.shape[1]
        s_loc = S // cp
        tt = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)
        wt = {k: (tt(v) if v is not None else None) for k, v in w.items()}
        bw = pkg.prepare_block_weights(wt, heads)
        kv = pkg.project_cross_kv(tt(ctx).to(torch.bfloat16), wt["attn2.k_proj_weight"], wt["attn2.k_proj_bias"],
                                  wt["attn2.norm_k.weight"], wt["attn2.v_proj_weight"], wt["attn2.v_proj_bias"], heads)
        cos_rh, sin_rh = rope.rope_rotate_half_caches(tt(cos).reshape(1, S, 1, 128), tt(sin).reshape(1, S, 1, 128))
        cos_rh, sin_rh = cos_rh.reshape(S, 128), sin_rh.reshape(S, 128)
        sl = slice(cp_rank * s_loc, (cp_rank + 1) * s_loc)
        h_bf = tt(hidden).to(torch.bfloat16)
        ring = pkg.wan_block_forward(h_bf[:, sl].contiguous(), tt(temb), (cos_rh[sl].contiguous(), sin_rh[sl].contiguous()),
                                     kv, bw, cp_size=cp, cp_group=None, cp_replica_groups=groups)
        full = pkg.wan_block_forward(h_bf, tt(temb), (cos_rh, sin_rh), kv, bw)
        torch.cuda.synchronize()
        got = ring.float().cpu().numpy().astype(np.float64)
        ref = full[:, sl].float().cpu().numpy().astype(np.float64)
        cos_sim = (got * ref).sum() / math.sqrt((got * got).sum() * (ref * ref).sum())
        res = (float(cos_sim), float(np.abs(got - ref).max()))
        pkg.destroy_rings()
        dist.destroy_process_group()
        out_q.put((rank, res, None))
    except Exception:
        out_q.put((rank, None, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs >= 4 GPUs")
def test_block_cfg_parallel_cp():
    world = 4
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_block_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for rank, r, tb in res:
        assert tb is None, tb
        cos_sim, mx = r
        assert cos_sim > 0.9999 and mx < 0.1, (rank, cos_sim, mx)
