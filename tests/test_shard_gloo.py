"""KV-head sharding of a long session on CPU ranks (gloo): each rank runs the
oracle decode for its heads, the outputs are all-gathered and reassembled, and
must equal the unsharded oracle bit for bit.  No GPU needed."""
import os

import numpy as np
import pytest

from llmhost_b200.shard import assemble, head_shard


def test_head_shard_ranges():
    s = [head_shard(r, 4, 8, 32) for r in range(4)]
    assert [(x.kv_begin, x.kv_end, x.q_begin, x.q_end) for x in s] == [(0, 2, 0, 8), (2, 4, 8, 16), (4, 6, 16, 24),
                                                                       (6, 8, 24, 32)]
    with pytest.raises(ValueError):
        head_shard(0, 3, 8, 32)


def _case(seed=0, n_tokens=700, n_q=32, n_kv=8, layers=2):
    from llmhost_b200.workloads import normal_bits

    rng = np.random.default_rng(seed)
    k = normal_bits(rng, (layers, n_tokens, n_kv, 64), "bf16")
    v = normal_bits(rng, (layers, n_tokens, n_kv, 64), "bf16")
    q = normal_bits(rng, (layers, n_q, 64), "bf16")
    return k, v, q


def _oracle_decode(k, v, q, n_q, n_kv):
    """One session, all layers: pages filled with the tokens, then decode at the last position."""
    from oracle import oracle as O

    layers, n, _, _ = k.shape
    pages = -(-n // 16)
    outs = []
    for layer in range(layers):
        host = O.HostPages(pages, O.BF16, n_q, n_kv)
        bt = np.arange(pages, dtype=np.uint32)
        for t in range(n):
            host.append_token(bt, t, t, np.ascontiguousarray(k[layer, t]), np.ascontiguousarray(v[layer, t]))
        outs.append(host.decode(bt, n, 0, np.ascontiguousarray(q[layer])))
    return np.stack(outs)  # [layers, n_q, d]


def _rank_main(rank, world, port, result):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n_q, n_kv = 32, 8
        k, v, q = _case()
        sh = head_shard(rank, world, n_kv, n_q)
        mine = _oracle_decode(k[:, :, sh.kv_begin:sh.kv_end], v[:, :, sh.kv_begin:sh.kv_end],
                              q[:, sh.q_begin:sh.q_end], sh.n_q, sh.n_kv)
        local = torch.from_numpy(mine)
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local)
        if rank == 0:
            result.put(assemble(torch.stack(parts)).numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_long_session_matches_unsharded(world):
    import multiprocessing as mp
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    k, v, qq = _case()
    want = _oracle_decode(k, v, qq, 32, 8)
    np.testing.assert_array_equal(got, want)
