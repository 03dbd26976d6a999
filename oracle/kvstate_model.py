"""Reference model of the KV state rules -- TEST INFRASTRUCTURE.

A plain-Python restatement, written separately from the C++ library, of
(1) the reference's tree rules (crates/llm-engine/src/tree.rs:41-123) and its
Engine bookkeeping (crates/llm-engine/src/batch.rs:128-297), and (2) the
build-defined page rules that the reference does not have (allocator order,
copy-on-write, draft fork, commit compaction, eviction, pool compaction):

* allocation pops a LIFO free stack seeded so the first page is order[0];
  a page goes back on top of the stack when its count drops to 0;
* operations walk layers 0..L-1 in order and each layer's pages in table order;
* a write into a partially filled tail page referenced elsewhere copies it first;
* forward forks a draft: token i -> slot base + i, RoPE position base + depth(i);
* commit moves accepted order[j] from slot base + order[j] to base + j, frees the
  draft's pages past ceil((base + a) / P) (from the end), releases the old tables
  (in order) and installs the draft;
* evict_window frees the pages wholly below n - window, in ascending order;
* compact moves each used page id >= U to the lowest free id (ascending) and
  re-seeds the free stack with U, U+1, ... next.

Tests drive this model and the library with the same operations and require
identical tables, free stacks, reference counts and plans.
"""
from __future__ import annotations

NONE = 0xFFFFFFFF


class TreeErr(Exception):
    def __init__(self, kind, a, b):
        self.kind, self.a, self.b = kind, a, b
        super().__init__(f"{kind}({a}, {b})")

    def key(self):
        return (self.kind, self.a, self.b)


def linear_tree(n):
    return [-1 if i == 0 else i - 1 for i in range(n)]


def validate_tree(tree):  # tree.rs:48-61
    for child, parent in enumerate(tree):
        if parent == -1:
            continue
        if parent < 0 or parent >= len(tree):
            raise TreeErr("ParentOutOfRange", child, parent)
        if parent >= child:
            raise TreeErr("ParentDoesNotPrecede", child, parent)


def validate_tree_for_tokens(tree, tokens):  # tree.rs:66-73
    if len(tree) != tokens:
        raise TreeErr("LengthMismatch", len(tree), tokens)
    validate_tree(tree)


def validate_accept_path(tree, accepted):  # tree.rs:90-123
    s = set(accepted)
    if len(s) != len(accepted):
        dup = next((i for i in accepted if accepted.count(i) > 1), 0)
        raise TreeErr("ParentDoesNotPrecede", dup, -2)
    for child in accepted:
        if child >= len(tree):
            raise TreeErr("ParentOutOfRange", child, child)
        parent = tree[child]
        if parent == -1:
            continue
        if parent < 0 or parent >= len(tree):
            raise TreeErr("ParentOutOfRange", child, parent)
        if parent not in s:
            raise TreeErr("ParentDoesNotPrecede", child, parent)


class ModelError(Exception):
    def __init__(self, kind, index=None):
        self.kind, self.index = kind, index
        super().__init__(kind)


class Model:
    def __init__(self, n_pages, n_layers, P=16, order=None):
        self.n_pages, self.L, self.P = n_pages, n_layers, P
        self.ref = [0] * n_pages
        seq = list(order) if order is not None else list(range(n_pages))
        self.free = list(reversed(seq))  # top = end
        self.sess = {}

    # allocator
    def alloc(self):
        p = self.free.pop()
        self.ref[p] = 1
        return p

    def decref(self, p):
        self.ref[p] -= 1
        if self.ref[p] == 0:
            self.free.append(p)

    def release(self, tables):
        for t in tables:
            for p in t:
                if p != NONE:
                    self.decref(p)

    def share(self, tables):
        for t in tables:
            for p in t:
                if p != NONE:
                    self.ref[p] += 1
        return [list(t) for t in tables]

    def need(self, tables, start, n):
        if n <= 0:
            return 0
        want = -(-(start + n) // self.P)
        k = 0
        for t in tables:
            if start % self.P and t[start // self.P] != NONE and self.ref[t[start // self.P]] > 1:
                k += 1
            k += max(0, want - len(t))
        return k

    def grow(self, tables, start, n, cow):
        if n <= 0:
            return
        want = -(-(start + n) // self.P)
        for t in tables:
            if start % self.P:
                i = start // self.P
                if t[i] != NONE and self.ref[t[i]] > 1:
                    fresh = self.alloc()
                    cow.append((t[i], fresh))
                    self.decref(t[i])
                    t[i] = fresh
            while len(t) < want:
                t.append(self.alloc())

    # sessions
    def _new(self):
        return {"tables": [[] for _ in range(self.L)], "n": 0, "committed": [], "pending": None}

    def open(self, seq):
        self.close(seq)
        self.sess[seq] = self._new()

    def close(self, seq):
        s = self.sess.pop(seq, None)
        if s is None:
            return
        if s["pending"]:
            self.release(s["pending"]["tables"])
        self.release(s["tables"])

    def fork(self, src, dst):
        if src not in self.sess:
            raise ModelError("UnknownSeq")
        if src == dst or dst in self.sess:
            raise ModelError("Invalid")
        s = self.sess[src]
        self.sess[dst] = {"tables": self.share(s["tables"]), "n": s["n"], "committed": list(s["committed"]),
                          "pending": None}

    def append(self, seq, n, tokens=None):
        if seq not in self.sess:
            raise ModelError("UnknownSeq")
        s = self.sess[seq]
        if n < 0 or s["pending"]:
            raise ModelError("Invalid")
        if self.need(s["tables"], s["n"], n) > len(self.free):
            raise ModelError("Oom")
        cow = []
        self.grow(s["tables"], s["n"], n, cow)
        s["n"] += n
        s["committed"] += list(tokens) if tokens is not None else [0] * n
        return cow

    def forward(self, seq, tokens, tree=None):
        tokens = list(tokens)
        t = list(tree) if tree is not None else linear_tree(len(tokens))
        if tree is not None:
            validate_tree_for_tokens(t, len(tokens))  # raises TreeErr
        if seq not in self.sess:
            self.sess[seq] = self._new()
        s = self.sess[seq]
        if s["pending"]:
            self.release(s["pending"]["tables"])
            s["pending"] = None
        d = {"tables": self.share(s["tables"]), "base": s["n"], "tokens": tokens, "tree": t}
        if self.need(d["tables"], d["base"], len(tokens)) > len(self.free):
            self.release(d["tables"])
            raise ModelError("Oom")
        cow = []
        self.grow(d["tables"], d["base"], len(tokens), cow)
        depth = []
        for p in t:
            depth.append(0 if p == -1 else depth[p] + 1)
        s["pending"] = d
        return [d["base"] + i for i in range(len(tokens))], [d["base"] + x for x in depth], cow

    def commit(self, seq, accepted):
        if seq not in self.sess:
            raise ModelError("UnknownSeq")
        s = self.sess[seq]
        d = s["pending"]
        if d is None:
            raise ModelError("NoPendingForward")
        try:
            validate_accept_path(d["tree"], accepted)
        except TreeErr as e:
            raise ModelError("InvalidAccept", accepted[0] if e.kind == "LengthMismatch" else e.a)
        for i in accepted:
            if i >= len(d["tokens"]):
                raise ModelError("InvalidAccept", i)
        order = sorted(set(accepted))
        a = len(order)
        moves = [(d["base"] + o, d["base"] + j) for j, o in enumerate(order) if o != j]
        keep = -(-(d["base"] + a) // self.P)
        for t in d["tables"]:
            for i in range(len(t) - 1, keep - 1, -1):
                if t[i] != NONE:
                    self.decref(t[i])
            del t[keep:]
        self.release(s["tables"])
        s["tables"] = d["tables"]
        s["committed"] += [d["tokens"][i] for i in order]
        s["n"] = d["base"] + a
        s["pending"] = None
        return moves

    def accept(self, seq, accepted):
        return self.commit(seq, list(accepted))

    def rollback(self, seq, rejected):
        if seq not in self.sess:
            raise ModelError("UnknownSeq")
        d = self.sess[seq]["pending"]
        if d is None:
            raise ModelError("NoPendingForward")
        rej = set(rejected)
        return self.commit(seq, [i for i in range(len(d["tokens"])) if i not in rej])

    def evict_window(self, seq, window):
        if seq not in self.sess:
            raise ModelError("UnknownSeq")
        s = self.sess[seq]
        if window <= 0 or s["pending"]:
            raise ModelError("Invalid")
        lo = max(0, s["n"] - window)
        k = 0
        for t in s["tables"]:
            for i in range(min(len(t), lo // self.P)):
                if t[i] != NONE:
                    self.decref(t[i])
                    t[i] = NONE
                    k += 1
        return k

    def compact(self):
        used = self.n_pages - len(self.free)
        holes = [p for p in range(used) if self.ref[p] == 0]
        movers = [p for p in range(used, self.n_pages) if self.ref[p] > 0]
        remap = {}
        for m, h in zip(movers, holes):
            remap[m] = h
            self.ref[h] = self.ref[m]
            self.ref[m] = 0
        if remap:
            for s in self.sess.values():
                groups = [s["tables"]] + ([s["pending"]["tables"]] if s["pending"] else [])
                for tables in groups:
                    for t in tables:
                        for i, p in enumerate(t):
                            if p != NONE and p in remap:
                                t[i] = remap[p]
        self.free = list(range(self.n_pages - 1, used - 1, -1))
        return list(zip(movers, holes))

    # views
    def free_list(self):
        return list(reversed(self.free))

    def table(self, seq, layer, draft=False):
        s = self.sess[seq]
        return list((s["pending"]["tables"] if draft else s["tables"])[layer])
