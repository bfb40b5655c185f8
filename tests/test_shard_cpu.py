"""KV-head sharding of a layer (palu_b200/shard.py) with world-size-2 gloo ranks on CPU.

Each rank slices its heads, runs the decode-attention oracle on its shard and multiplies by its block of
``wo_fused``; the all-reduced sum must equal the unsharded layer tail (concat heads @ wo_fused^T,
palu_tt/attention.py:718-733). M-LRD (absorbed V) and G-LRD (V rebuilt per head, 2 groups) are covered.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from oracle.metrics import rel_errors

THETA = 500000.0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer(seed, grouped):
    g = torch.Generator().manual_seed(seed)
    B, n_q, n_kv, S, dim = 2, 8, 4, 96, 256
    n_groups, r = (2, 32) if grouped else (4, 16)
    bf = lambda t: t.to(torch.bfloat16).float()
    q = bf(torch.randn(B, n_q, 128, generator=g))
    k_lat = bf(torch.randn(B, n_groups, S, r, generator=g))
    v_lat = bf(torch.randn(B, n_groups, S, r, generator=g))
    u_k = bf(torch.randn(n_kv, r, 128, generator=g) / r ** 0.5)
    u_v = bf(torch.randn(n_kv, r, 128, generator=g) / r ** 0.5) if grouped else None
    wo = torch.randn(dim, n_q * 128, generator=g) / (n_q * 128) ** 0.5
    pos = torch.tensor([S - 1, S // 3])
    cos, sin = oracle.cos_sin_tables(128, S, THETA, None)
    return dict(q=q, k_lat=k_lat, v_lat=v_lat, u_k=u_k, u_v=u_v, wo=wo, pos=pos, cos=cos[:S], sin=sin[:S],
                n_q=n_q, n_kv=n_kv, n_groups=n_groups)


def _attend(q, k_lat, v_lat, u_k, u_v, pos, cos, sin, n_kv):
    gs = n_kv // k_lat.shape[1]  # KV heads per latent group
    k = oracle.expand_groups(k_lat, gs)
    v = oracle.expand_groups(v_lat, gs)
    return oracle.reference_decode(q[None], k, u_k, v, pos, cos, sin, 128 ** -0.5, u_v=u_v)[0]


def _unsharded(L):
    o = _attend(L["q"], L["k_lat"], L["v_lat"], L["u_k"], L["u_v"], L["pos"], L["cos"], L["sin"], L["n_kv"])
    from palu_b200.shard import layer_output_partial
    return layer_output_partial(o, L["wo"])


def _rank_main(rank, world, port, grouped, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "tt-cadlab_b200")]
    from palu_b200.shard import KVShard, all_reduce_layer_output, layer_output_partial, shard_layer_inputs
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        L = _layer(7, grouped)
        sh = KVShard(rank, world, L["n_kv"], L["n_q"], L["n_groups"])
        x = shard_layer_inputs(sh, L["q"], L["k_lat"], L["v_lat"], L["u_k"], L["wo"], L["u_v"])
        o = _attend(x["q"], x["k_lat"], x["v_lat"], x["u_k"], x["u_v"], L["pos"], L["cos"], L["sin"],
                    len(sh.kv))
        part = all_reduce_layer_output(layer_output_partial(o, x["wo"]))
        if rank == 0:  # a numpy array travels by value (a shared-memory tensor can race this process's exit)
            out_q.put(part.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("grouped,world", [(False, 2), (True, 2), (True, 4)], ids=["mlrd", "glrd", "glrd_split4"])
def test_sharded_layer_equals_unsharded(grouped, world):
    """2 ranks: heads and whole latent groups split; 4 ranks with 2 groups: each group's heads split over
    two ranks, each holding the whole group latent."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, grouped, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = torch.from_numpy(q.get(timeout=90))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = _unsharded(_layer(7, grouped))
    mx, mn = rel_errors(got, want)
    assert mx < 1e-5 and mn < 1e-5, (mx, mn)


def test_shard_ranges_cover_every_head_once():
    from palu_b200.shard import KVShard
    for world in (1, 2, 4, 8):
        shards = [KVShard(r, world, 8, 32, 8) for r in range(world)]
        assert sorted(h for s in shards for h in s.kv) == list(range(8))
        assert sorted(h for s in shards for h in s.q) == list(range(32))
    # 2 G-LRD groups over 4 or 8 ranks: each group's heads split, its latent replicated on those ranks
    for world in (4, 8):
        shards = [KVShard(r, world, 8, 32, 2) for r in range(world)]
        assert sorted(h for s in shards for h in s.kv) == list(range(8))
        for s in shards:
            assert list(s.groups) == [s.kv.start // 4] and s.kv.stop - 1 < 4 * (s.kv.start // 4 + 1)
            assert s.latent_replicas == world // 2
    assert KVShard(0, 2, 8, 32, 2).latent_replicas == 1
    with pytest.raises(ValueError, match="do not shard"):
        KVShard(0, 3, 6, 24, 2)  # neither 2 groups nor 3 ranks divides the other
