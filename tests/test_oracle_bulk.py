"""The oracle's bulk helpers against its per-token restatement (no GPU needed).

The full-size parity tests fill pages and run prefill / tree-verify attention
through orc_paged_append_tokens and orc_paged_prefill (threaded), and decode
under a window through the windowed gather of orc_paged_decode.  Each must give
the same bits as the plain restatement it stands for:

* append_tokens == one orc_paged_append_token call per token;
* prefill == gather + RoPE + orc_attention_masked with the explicit mask
  (attention_forward's loop, lfm2.rs:1058-1111);
* a windowed decode == attention_decode_cached (lfm2.rs:1006-1056) over the
  whole row with keys below the window masked through key_valid.
"""
import numpy as np
import pytest

from llmhost_b200.plans import tree_masks
from llmhost_b200.workloads import normal_bits
from oracle import oracle as O

NONE = 0xFFFFFFFF


def _tables(rng, lens, n_pages):
    pages = -(-np.asarray(lens) // 16)
    perm = rng.permutation(n_pages).astype(np.uint32)
    bt = np.full((len(lens), max(int(pages.max()), 1)), NONE, np.uint32)
    cur = 0
    for s, p in enumerate(pages):
        bt[s, :p] = perm[cur:cur + p]
        cur += p
    return bt


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_append_tokens_equals_per_token_appends(dtype):
    rng = np.random.default_rng(1)
    lens = [0, 5, 16, 37, 300]
    n_pages = sum(-(-x // 16) for x in lens) + 3
    bt = _tables(rng, lens, n_pages)
    n_kv = 8
    odt = O.BF16 if dtype == "bf16" else O.F32
    a = O.HostPages(n_pages, odt, 24, n_kv)
    b = O.HostPages(n_pages, odt, 24, n_kv)
    rows = np.concatenate([np.full(x, s, np.int32) for s, x in enumerate(lens)])
    slots = np.concatenate([np.arange(x, dtype=np.int32) for x in lens])
    pos = slots * 3 + 7  # RoPE positions need not equal slots
    k = normal_bits(rng, (len(slots), n_kv, 64), dtype)
    v = normal_bits(rng, (len(slots), n_kv, 64), dtype)
    for i in range(len(slots)):
        a.append_token(bt[rows[i]], int(slots[i]), int(pos[i]), k[i], v[i])
    b.append_tokens(bt, rows, slots, pos, k, v, n_threads=4)
    np.testing.assert_array_equal(a.data, b.data)


@pytest.mark.parametrize("tree", [False, True])
@pytest.mark.parametrize("n_q,n_kv", [(24, 8), (8, 2)])
def test_paged_prefill_equals_masked_attention(tree, n_q, n_kv):
    rng = np.random.default_rng(2 + n_q + tree)
    cached = [0, 19, 64, 130]
    if tree:
        parents = [[-1] + [int(rng.integers(0, i)) for i in range(1, T)] for T in (1, 9, 20, 33)]
        T = [len(p) for p in parents]
    else:
        T = [7, 1, 40, 0]
    tot = [c + t for c, t in zip(cached, T)]
    n_pages = sum(-(-x // 16) for x in tot) + 2
    bt = _tables(rng, tot, n_pages)
    host = O.HostPages(n_pages, O.BF16, n_q, n_kv)
    rows = np.concatenate([np.full(x, s, np.int32) for s, x in enumerate(tot)])
    slots = np.concatenate([np.arange(x, dtype=np.int32) for x in tot])
    pos = slots.copy()
    if tree:  # a draft token's RoPE position is prefix + its depth
        off = 0
        for s, (c, p) in enumerate(zip(cached, parents)):
            depth = []
            for x in p:
                depth.append(0 if x < 0 else depth[x] + 1)
            pos[off + c:off + c + len(p)] = c + np.array(depth)
            off += c + len(p)
    k = normal_bits(rng, (len(slots), n_kv, 64), "bf16")
    v = normal_bits(rng, (len(slots), n_kv, 64), "bf16")
    host.append_tokens(bt, rows, slots, pos, k, v)
    q_off = np.concatenate([[0], np.cumsum(T)]).astype(np.int32)
    q_pos = np.concatenate([pos[rows == s][c:] for s, c in enumerate(cached)]).astype(np.int32)
    q = normal_bits(rng, (int(q_off[-1]), n_q, 64), "bf16")
    masks = np.concatenate([tree_masks(p) for p in parents]) if tree else None
    got = host.prefill(bt, cached, q_off, q_pos, q, masks=masks, n_threads=3)
    for s in range(len(cached)):
        L, t = cached[s], T[s]
        if t == 0:
            continue
        kk, vv = host.gather(bt[s], L + t)
        qf = O.bf16_bits_to_f32(q[q_off[s]:q_off[s + 1]]).copy()
        for i in range(t):
            c, sn = O.cos_sin(host.inv, int(q_pos[q_off[s] + i]), 1, 64)
            O.apply_rope_in_place(qf[i], c, sn, n_q, 1, 64)
        mask = np.zeros((t, L + t), np.uint8)
        mask[:, :L] = 1
        for i in range(t):
            if tree:
                bits = int(masks[q_off[s] + i].view(np.uint64))
                mask[i, L:] = [(bits >> j) & 1 for j in range(t)]
            else:
                mask[i, L:L + i + 1] = 1
        ref = O.attention_masked(np.ascontiguousarray(qf.transpose(1, 0, 2)), kk, vv, n_q, n_kv, t, L + t, 64, mask)
        np.testing.assert_array_equal(got[q_off[s]:q_off[s + 1]], ref.transpose(1, 0, 2))


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("seq_len,window", [(1, 4), (100, 16), (100, 100), (100, 99), (517, 33), (2000, 1024)])
def test_windowed_decode_equals_masked_row(dtype, seq_len, window):
    rng = np.random.default_rng(seq_len + window)
    n_q, n_kv = 24, 8
    n_pages = -(-seq_len // 16) + 1
    bt = _tables(rng, [seq_len], n_pages)[0]
    odt = O.BF16 if dtype == "bf16" else O.F32
    host = O.HostPages(n_pages, odt, n_q, n_kv)
    slots = np.arange(seq_len, dtype=np.int32)
    host.append_tokens(bt, np.zeros(seq_len, np.int32), slots, slots,
                       normal_bits(rng, (seq_len, n_kv, 64), dtype), normal_bits(rng, (seq_len, n_kv, 64), dtype))
    q = normal_bits(rng, (n_q, 64), dtype)
    got = host.decode(bt, seq_len, window, q)
    # the reference's masked row: every key gathered, keys below the window masked
    k, v = host.gather(bt, seq_len)
    qf = (O.bf16_bits_to_f32(q) if dtype == "bf16" else q).copy()
    c, sn = O.cos_sin(host.inv, seq_len - 1, 1, 64)
    O.apply_rope_in_place(qf, c, sn, n_q, 1, 64)
    valid = (np.arange(seq_len) + window >= seq_len).astype(np.uint8)
    ref = O.attention_decode_cached(qf, k, v, n_q, n_kv, seq_len, seq_len, 64, key_valid=valid)
    np.testing.assert_array_equal(got, ref)
