"""Context-parallel ring of the const-max attention (host side of ``vomni_ring_*``).

Mirrors the reference's ring contract: ``replica_groups`` lists every ring as a tuple of global ranks
(``get_cp_replica_groups``, vllm_omni_neuron/diffusion/distributed/parallel_state.py:180-188) and each
SPMD rank resolves its own ring; ``num_workers`` is the CP degree; every rank of a ring calls the
attention collectively, in the same order (ring_attention_const_max_fwd.py:958-1017).

A ring context (NCCL communicator, IPC-registered send buffer, gather buffer, workspace) is created
once per (process group, b, h) and grown when a longer shard arrives — the analogue of the
reference's one-time replica-group registration (parallel_state.py:355-415). Creation and growth
are collective; every rank sees the same shapes, so they happen on all ranks together.
"""

from __future__ import annotations

import ctypes
import math

import torch
import torch.distributed as dist

from . import _lib

_RINGS: dict = {}
_SUBGROUPS: dict = {}


class RingContext:
    def __init__(self, group, b: int, s_max: int, h: int, d: int):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.b, self.s_max, self.h, self.d = b, s_max, h, d
        L = _lib.load()
        uid = ctypes.create_string_buffer(128)
        if self.rank == 0:
            _lib.check(L.vomni_nccl_unique_id(uid, 128), "vomni_nccl_unique_id")
        obj = [uid.raw if self.rank == 0 else None]
        src = dist.get_global_rank(group, 0) if group is not dist.group.WORLD else 0
        dist.broadcast_object_list(obj, src=src, group=group)
        uid = ctypes.create_string_buffer(obj[0], 128)
        self.handle = ctypes.c_void_p()
        _lib.check(
            L.vomni_ring_create(ctypes.byref(self.handle), self.rank, self.world, uid, 128, b, s_max, h, d),
            "vomni_ring_create",
        )

    def close(self):
        if self.handle:
            _lib.load().vomni_ring_destroy(self.handle)
            self.handle = ctypes.c_void_p()

    def check(self):
        _lib.check(_lib.load().vomni_ring_check(self.handle), "vomni_ring_check")


def _group_for(replica_groups, num_workers: int):
    """The process group of this rank's ring. ``replica_groups=None`` means the whole world."""
    if not dist.is_available() or not dist.is_initialized():
        raise RuntimeError("num_workers > 1 needs an initialised torch.distributed process group")
    if not replica_groups:
        assert dist.get_world_size() == num_workers, (
            f"num_workers={num_workers} but the default group has {dist.get_world_size()} ranks; pass replica_groups"
        )
        return dist.group.WORLD
    key = tuple(tuple(int(r) for r in g) for g in replica_groups)
    if key not in _SUBGROUPS:
        me = dist.get_rank()
        mine = None
        for ranks in key:  # new_group is collective over the world: create every ring, in order
            g = dist.new_group(list(ranks))
            if me in ranks:
                mine = g
        if mine is None:
            raise RuntimeError(f"rank {me} is in none of the replica groups {key}")
        _SUBGROUPS[key] = mine
    return _SUBGROUPS[key]


def get_ring(group, b: int, s_loc: int, h: int, d: int) -> RingContext:
    key = (id(group), b, h, d)
    r = _RINGS.get(key)
    if r is None or r.s_max < s_loc:
        if r is not None:
            torch.cuda.synchronize()
            r.close()
        r = RingContext(group, b, s_loc, h, d)
        _RINGS[key] = r
    return r


def destroy_rings():
    """Release every ring context (call before ``destroy_process_group``)."""
    if _RINGS:
        torch.cuda.synchronize()
    for r in _RINGS.values():
        r.close()
    _RINGS.clear()


def ring_attention(
    q, k, v, *, replica_groups, num_workers, softmax_scale, training, kv_prefetch_depth, group, out_layout
):
    b, s, h, d = q.shape
    if group is None:
        group = _group_for(replica_groups, num_workers)
    world = dist.get_world_size(group)
    assert world == num_workers, f"num_workers={num_workers} does not match the ring's {world} ranks"
    # kv_prefetch_depth is clamped as the reference does (:1078); the copy engine pulls every block
    # as soon as the key max is reduced, and the pass plan gates compute on arrival.
    _ = min(max(int(kv_prefetch_depth), 1), max(num_workers - 1, 1))
    from .attention import token_major

    q, q_stride = token_major(q)
    k, k_stride = token_major(k)
    v, v_stride = token_major(v)
    if k_stride != v_stride:
        k, v = k.contiguous(), v.contiguous()
        k_stride = h * d
    ring = get_ring(group, b, s, h, d)
    scale = float(softmax_scale) if softmax_scale else 1.0 / math.sqrt(d)
    flags = 0
    if out_layout == "bhds":
        flags |= _lib.CM_OUT_DMAJOR
        out = torch.empty((b, h, d, s), dtype=torch.bfloat16, device=q.device)
    elif out_layout == "bhsd":
        out = torch.empty((b, h, s, d), dtype=torch.bfloat16, device=q.device)
    else:
        raise ValueError(f"unknown out_layout {out_layout!r}")
    lse = None
    if training:
        flags |= _lib.CM_LSE
        lse = torch.zeros((b, h, 128, -(-s // 128)), dtype=torch.float32, device=q.device)
    rc = _lib.load().vomni_ring_attention_strided(
        ring.handle, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
        lse.data_ptr() if lse is not None else None, b, s, h, d, q_stride, k_stride, scale, flags,
        torch.cuda.current_stream(q.device).cuda_stream,
    )
    _lib.check(rc, "vomni_ring_attention_strided")
    return (out, lse) if training else out


def phase_plan(world: int):
    """(first, count) of each pass; pass 0 is the local block (first = -1)."""
    L = _lib.load()
    first = (ctypes.c_int * 64)()
    count = (ctypes.c_int * 64)()
    n = L.vomni_ring_phase_plan(world, first, count, 64)
    if n < 0:
        raise ValueError(f"bad world size {world}")
    return [(first[i], count[i]) for i in range(n)]


def source_rank(rank: int, world: int, step: int) -> int:
    return _lib.load().vomni_ring_source_rank(rank, world, step)
