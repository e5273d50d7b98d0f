"""CPU tests of the ring's host logic: the pass plan and ring order (through the C ABI, host-only
functions) and a world-size-2 gloo emulation of the ring schedule against the oracle. No GPU."""

import os
import socket
import traceback

import numpy as np
import pytest
import torch.multiprocessing as mp


@pytest.fixture(scope="module")
def ring(pkg):
    from importlib import import_module

    return import_module("vllm-omni-neuron_b200.ring")


@pytest.mark.parametrize("world", [1, 2, 3, 4, 5, 8, 16])
def test_phase_plan_covers_each_block_once(ring, world):
    plan = ring.phase_plan(world)
    assert plan[0] == (-1, 1)  # pass 0 = local block
    slots = []
    size = 1
    for first, count in plan[1:]:
        assert first == len(slots)
        assert 1 <= count <= size
        slots.extend(range(first, first + count))
        size *= 2
    assert slots == list(range(world - 1))


def test_phase_plan_default(ring):
    """The pass sizes double after the local pass: 1, 2, 4, ... (the last pass takes the remainder)."""
    assert ring.phase_plan(8) == [(-1, 1), (0, 1), (1, 2), (3, 4)]
    assert ring.phase_plan(4) == [(-1, 1), (0, 1), (1, 2)]
    assert ring.phase_plan(1) == [(-1, 1)]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_ring_order(ring, world):
    for r in range(world):
        srcs = [ring.source_rank(r, world, s) for s in range(world)]
        assert srcs[0] == r
        assert sorted(srcs) == list(range(world))
        # step s consumes what rank r-1 consumed at step s-1 (forward-to-next-rank ring)
        for s in range(1, world):
            assert srcs[s] == ring.source_rank((r - 1) % world, world, s - 1)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard(rank, b=1, s=96, h=2, seed=11):
    from oracle.numerics import bf16_round

    rng = np.random.default_rng(seed + rank)
    return [bf16_round(rng.standard_normal((b, s, h, 128)).astype(np.float32) * 0.7) for _ in range(3)]


def _emulated_ring_worker(rank, world, port, out_q, fault=None):
    try:
        import torch
        import torch.distributed as dist

        from importlib import import_module

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from oracle import attention as oat

        ring = import_module("vllm-omni-neuron_b200.ring")
        q, k, v = _shard(rank)
        scale = 1 / np.sqrt(128)
        # local norms, then the global key max by all_reduce(max) — as the ring does with NCCL
        qn2 = np.einsum("bshd,bshd->bhs", q, q)
        kmax = torch.from_numpy(np.einsum("bshd,bshd->bhs", k, k).max(axis=-1).copy())
        dist.all_reduce(kmax, op=dist.ReduceOp.MAX)
        c = oat.bf16_round(np.sqrt(np.float32(scale) ** 2 * kmax.numpy()[:, :, None] * qn2))
        # the peer copies: every rank's K/V block (all_gather stands in for the IPC pulls)
        ks = [torch.zeros(k.shape) for _ in range(world)]
        vs = [torch.zeros(v.shape) for _ in range(world)]
        dist.all_gather(ks, torch.from_numpy(k))
        dist.all_gather(vs, torch.from_numpy(v))
        # gather buffer in ring-step order: slot j holds step j+1's block
        src = (lambda s: (rank + s) % world) if fault == "order" else (lambda s: ring.source_rank(rank, world, s))
        gk = np.concatenate([ks[src(s)].numpy() for s in range(1, world)], axis=1)
        gv = np.concatenate([vs[src(s)].numpy() for s in range(1, world)], axis=1)
        acc, ssum = oat.const_max_partial(q, k, v, c, scale)  # pass 0: local block
        s_loc = q.shape[1]
        plan = ring.phase_plan(world)[1:]
        if fault == "drop":  # the last pass loses its last block
            first, count = plan[-1]
            plan = plan[:-1] + ([(first, count - 1)] if count > 1 else [])
        if fault == "dup":  # the first remote block is accumulated twice
            plan = plan + [plan[0]]
        for first, count in plan:
            sl = slice(first * s_loc, (first + count) * s_loc)
            a, sm = oat.const_max_partial(q, gk[:, sl], gv[:, sl], c, scale)
            acc += a
            ssum += sm
        o = oat.const_max_normalize(acc, ssum)
        ref = oat.const_max_ring_attention([_shard(r)[0] for r in range(world)], [_shard(r)[1] for r in range(world)],
                                           [_shard(r)[2] for r in range(world)], scale)[rank]
        exact = oat.wan_cp_self_attention_oracle([_shard(r)[0] for r in range(world)], [_shard(r)[1] for r in range(world)],
                                                 [_shard(r)[2] for r in range(world)], scale)[rank]
        err_ring = float(np.abs(o - ref).max())
        err_exact = float(np.abs(np.transpose(o, (0, 1, 3, 2)) - exact).max())
        dist.destroy_process_group()
        out_q.put((rank, err_ring, err_exact, None))
    except Exception:
        out_q.put((rank, None, None, traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 3])
def test_ring_schedule_gloo(ring, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_emulated_ring_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, e_ring, e_exact, tb in res:
        assert tb is None, tb
        # pass order differs from the step order only by fp32 summation order
        assert e_ring <= 1e-2, (rank, e_ring)
        assert e_exact <= 2e-2, (rank, e_exact)


@pytest.mark.parametrize("world,fault", [(2, "drop"), (3, "drop"), (3, "dup"), (3, "order")])
def test_ring_schedule_faults_gloo(ring, world, fault):
    """Faults planted in the emulated schedule: a dropped or duplicated K/V block is caught by the
    comparison with the oracle; a wrong rotation direction (each remote block still used once) gives
    the right result, because const-max partials combine by plain addition in any order."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_emulated_ring_worker, args=(r, world, port, q, fault)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, e_ring, e_exact, tb in res:
        assert tb is None, tb
        if fault == "order":
            assert e_ring <= 1e-2 and e_exact <= 2e-2, (rank, e_ring, e_exact)
        else:
            assert e_ring > 5e-2 and e_exact > 5e-2, (rank, fault, e_ring, e_exact)


def _dying_rank_worker(rank, world, port, out_q):
    """Rank 1 fails before the collective; rank 0 must get an error from a short timeout, not hang."""
    try:
        from datetime import timedelta

        import torch
        import torch.distributed as dist

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
        if rank == 1:
            raise RuntimeError("injected failure before the key-max all_reduce")
        t = torch.ones(4)
        try:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            out_q.put((rank, "no error"))
        except Exception as e:  # timeout / connection reset surface here
            out_q.put((rank, f"error: {type(e).__name__}"))
    except RuntimeError as e:
        out_q.put((rank, f"raised: {e}"))


def test_rank_failure_surfaces_as_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert res[1].startswith("raised")
    assert res[0].startswith("error"), res[0]


def _cp_shard_gather_worker(rank, world, port, q):
    try:
        import os
        from importlib import import_module

        import torch
        import torch.distributed as dist

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        dit = import_module("vllm-omni-neuron_b200.dit")
        g = torch.Generator().manual_seed(0)
        hidden = torch.randn(2, 12 * world, 8, generator=g)
        cos = torch.randn(1, 12 * world, 1, 16, generator=g)
        sin = torch.randn(1, 12 * world, 1, 16, generator=g)
        local, (lc, ls) = dit.cp_shard_sequence(hidden, (cos, sin), rank, world)
        ok = torch.equal(local, hidden[:, rank * 12:(rank + 1) * 12]) and torch.equal(lc, cos[:, rank * 12:(rank + 1) * 12])
        back = dit.cp_gather_sequence(local * 2)
        ok = ok and torch.equal(back, hidden * 2)
        try:
            dit.cp_shard_sequence(hidden[:, :-1], None, rank, world)
            ok = ok and world == 1
        except ValueError:
            pass
        dist.destroy_process_group()
        q.put((rank, ok, None))
    except Exception:
        import traceback

        q.put((rank, False, traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 3])
def test_cp_shard_gather_gloo(world):
    """The DiT-level CP split / all-gather (wan2_2_transformer.py:1774-1831) on gloo ranks."""
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_cp_shard_gather_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, tb in res:
        assert tb is None, tb
        assert ok, rank


def _cfg_host_worker(rank, world, port, q):
    try:
        import os
        from importlib import import_module

        import torch
        import torch.distributed as dist

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        cfg = import_module("vllm-omni-neuron_b200.cfg")
        x = torch.full((4, 8), float(rank), dtype=torch.bfloat16)
        outcome = None
        try:
            cfg.cfg_gather_combine(x, 5.0)
        except ValueError:
            outcome = "world"  # a CFG group must have two ranks
        except RuntimeError:
            outcome = "no_cpu_path"  # gathered on gloo, then the GPU combine refuses CPU tensors
        try:
            cfg.cfg_gather_combine((x, x), 5.0)
            tuple_ok = False
        except (NotImplementedError, ValueError):
            tuple_ok = True
        dist.destroy_process_group()
        q.put((rank, outcome, tuple_ok, None))
    except Exception:
        import traceback

        q.put((rank, None, False, traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 3])
def test_cfg_gather_combine_host_checks(world):
    """CFG gather + combine host logic on gloo ranks (cfg_parallel.py:48-71, 135-159): a group other
    than two ranks is refused, a tuple branch output is refused, and the combine has no CPU path."""
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_cfg_host_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, outcome, tuple_ok, tb in res:
        assert tb is None, tb
        assert outcome == ("no_cpu_path" if world == 2 else "world"), (rank, outcome)
        assert tuple_ok, rank
