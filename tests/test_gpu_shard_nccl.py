"""KV-head sharding of one long session over 2 GPUs with NCCL.

The long-context configuration's 1M-token session is split by KV head: each
rank holds its KV heads' pages and their query heads, runs the fused decode
step for them, and one all_gather_into_tensor per step (every layer at once)
reassembles the heads.  Here a 131 072-token session of 32q/8kv, two layers:
rank r of 2 decodes KV heads 4r..4r+3 (the 16q/4kv kernel), NCCL gathers the
outputs, and rank 0 checks them against the CPU oracle and against one GPU
decoding all eight heads (the 32q/8kv kernel).  The two kernels cut the keys
into different splits, so the comparison is within the bf16 tolerance, not
bit for bit; the stored pages of each rank are bit-identical to the oracle's.
Skipped with fewer than two GPUs.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N_TOK, LAYERS, N_Q, N_KV, WORLD = 131072, 2, 32, 8, 2


def _data():
    from llmhost_b200.workloads import normal_bits

    rng = np.random.default_rng(77)
    k = normal_bits(rng, (LAYERS, N_TOK, N_KV, 64), "bf16")
    v = normal_bits(rng, (LAYERS, N_TOK, N_KV, 64), "bf16")
    q = normal_bits(rng, (LAYERS, N_Q, 64), "bf16")
    order = rng.permutation(N_TOK // 16 + 8).astype(np.uint32)
    return k, v, q, order


def _sample_ids(bt):
    """The page ids whose contents are compared: the 64 lowest and 64 highest
    of the session (the decode token's page among them when it is)."""
    ids = np.sort(bt)
    return np.unique(np.concatenate([ids[:64], ids[-64:], bt[-1:]]))


def _decode(dev, k, v, q, order, n_q, n_kv):
    """Fill one session's pages (all tokens but the last), then one fused decode
    step per layer.  Returns outputs [layers, n_q, 64] (bf16 bits) and the pages."""
    import torch
    from llmhost_b200.kv import KvPool

    n_pages = len(order)
    bt = order[:N_TOK // 16][None, :]
    outs, pages = [], []
    with KvPool(dtype="bf16", n_q_heads=n_q, n_kv_heads=n_kv, n_pages=n_pages, max_positions=N_TOK + 16, max_seqs=1,
                device=dev.index) as pool:
        bt_d = torch.from_numpy(bt.view(np.int32)).to(dev)
        pos = torch.arange(N_TOK - 1, dtype=torch.int32, device=dev)
        zero = torch.zeros(N_TOK - 1, dtype=torch.int32, device=dev)
        lens = torch.tensor([N_TOK], dtype=torch.int32, device=dev)

        def t(bits):
            return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(dev)

        for layer in range(LAYERS):
            pool.append(t(k[layer, :-1]), t(v[layer, :-1]), zero, pos, pos, bt_d)
            out = pool.append_decode_attn(t(k[layer, -1:]), t(v[layer, -1:]), t(q[layer][None]), bt_d, lens)
            torch.cuda.synchronize(dev)
            assert pool.last_error() == 0
            outs.append(out[0])
            pages.append(pool.read_pages(_sample_ids(bt[0])))
    return torch.stack(outs), pages


def _rank_main(rank, port, result):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from llmhost_b200.shard import assemble, head_shard

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=timedelta(seconds=120), device_id=dev)
    try:
        k, v, q, order = _data()
        sh = head_shard(rank, WORLD, N_KV, N_Q)
        mine, pages = _decode(dev, np.ascontiguousarray(k[:, :, sh.kv_begin:sh.kv_end]),
                              np.ascontiguousarray(v[:, :, sh.kv_begin:sh.kv_end]),
                              np.ascontiguousarray(q[:, sh.q_begin:sh.q_end]), order, sh.n_q, sh.n_kv)
        gathered = torch.empty((WORLD,) + tuple(mine.shape), dtype=mine.dtype, device=dev)
        dist.all_gather_into_tensor(gathered, mine.contiguous())
        torch.cuda.synchronize(dev)
        full = assemble(gathered).float().cpu().numpy()
        result.put((rank, "pages", pages))
        if rank == 0:
            whole, _ = _decode(dev, k, v, q, order, N_Q, N_KV)
            result.put((rank, "out", full, whole.float().cpu().numpy()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_head_sharded_session_nccl_allgather_matches_one_gpu_and_oracle():
    import multiprocessing as mp
    import socket

    import torch

    from oracle import oracle as O
    from paged_case import assert_close_rows

    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q_res = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, port, q_res)) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(WORLD + 1):
            item = q_res.get(timeout=600)
            got[(item[0], item[1])] = item[2:]
    finally:
        for p in procs:
            p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]

    k, v, q, order = _data()
    bt = order[:N_TOK // 16]
    ids = _sample_ids(bt)
    sharded, whole = got[(0, "out")]
    for layer in range(LAYERS):
        host = O.HostPages(len(order), O.BF16, N_Q, N_KV)
        slots = np.arange(N_TOK, dtype=np.int32)
        host.append_tokens(bt, np.zeros(N_TOK, np.int32), slots, slots, k[layer], v[layer])
        ref = host.decode(bt, N_TOK, 0, q[layer])
        assert_close_rows(sharded[layer], ref, 2e-2, f"sharded layer {layer} vs oracle")
        assert_close_rows(whole[layer], ref, 2e-2, f"one GPU layer {layer} vs oracle")
        assert_close_rows(sharded[layer], whole[layer], 2e-2, f"sharded vs one GPU, layer {layer}")
        # each rank's pages hold exactly its KV heads' K and V rows of the oracle's pages
        pages = host.data[ids].reshape(len(ids), 2, N_KV, 16, 64)
        for r in range(WORLD):
            per = N_KV // WORLD
            want = pages[:, :, r * per:(r + 1) * per].reshape(len(ids), -1)
            np.testing.assert_array_equal(got[(r, "pages")][0][layer], want, err_msg=f"rank {r} pages, layer {layer}")
