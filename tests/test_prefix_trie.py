"""The engine's prefix trie and block book replayed against the reference's
RadixCache / PagedCache (core/include/tvara/radix.hpp:17-130, kv.hpp:36-165)
compiled from its own sources: after every random operation both hold the same
node ids, lookup and reuse results, return codes, reference counts, free-block
count and block tables.  Needs no GPU."""

import ctypes as C

import numpy as np
import pytest


def _i32(tokens):
    return np.ascontiguousarray(tokens, dtype=np.int32)


class Ours:
    def __init__(self, L, blocks, tpb):
        self.L, self.b, self.blocks = L, L.tvara_kv_book_new(1, 1, 4, tpb, blocks), blocks

    def create(self):
        return self.L.tvara_kv_book_create(self.b)

    def append(self, s):
        return self.L.tvara_kv_book_append(self.b, s)

    def drop(self, s):
        return self.L.tvara_kv_book_drop(self.b, s)

    def fork(self, s):
        return self.L.tvara_kv_book_fork(self.b, s)

    def truncate(self, s, n):
        return self.L.tvara_kv_book_truncate(self.b, s, n)

    def insert(self, toks):
        t = _i32(toks)
        return self.L.tvara_kv_book_prefix_insert(self.b, t.ctypes.data_as(C.POINTER(C.c_int32)), len(t))

    def attach(self, node, s):
        return self.L.tvara_kv_book_prefix_attach(self.b, node, s)

    def lookup(self, toks):
        t = _i32(toks)
        node, n = C.c_uint64(), C.c_size_t()
        assert self.L.tvara_kv_book_prefix_lookup(self.b, t.ctypes.data_as(C.POINTER(C.c_int32)), len(t),
                                                  C.byref(node), C.byref(n)) == 0
        return node.value, n.value

    def reuse(self, toks, partial):
        t = _i32(toks)
        n = C.c_size_t()
        s = self.L.tvara_kv_book_prefix_reuse(self.b, t.ctypes.data_as(C.POINTER(C.c_int32)), len(t), partial,
                                              C.byref(n))
        return s, n.value

    def node_op(self, name, node):
        return getattr(self.L, "tvara_kv_book_prefix_" + name)(self.b, node)

    def evict(self):
        return self.L.tvara_kv_book_prefix_evict_one(self.b)

    def state(self, live):
        tables = {}
        for s in live:
            ids, gens, n = (C.c_uint64 * 4096)(), (C.c_uint64 * 4096)(), C.c_size_t()
            assert self.L.tvara_kv_book_table(self.b, s, ids, gens, 4096, C.byref(n)) == 0
            tables[s] = [(ids[i], gens[i]) for i in range(n.value)]
        return (self.L.tvara_kv_book_available(self.b),
                [self.L.tvara_kv_book_references(self.b, i) for i in range(self.blocks)],
                tables, self.L.tvara_kv_book_prefix_size(self.b))

    def audit(self):
        return self.L.tvara_kv_book_audit(self.b)


class Ref:
    def __init__(self, R, blocks, tpb):
        self.R, self.c, self.blocks = R, R.ref_cache_new(1, 1, 4, tpb, blocks), blocks
        assert R.ref_radix_new(self.c, b"replay") == 0
        self.x = np.zeros(4, np.float32)

    def create(self):
        return self.R.ref_cache_create(self.c)

    def append(self, s):
        return self.R.ref_cache_append(self.c, s, self.x, self.x)

    def drop(self, s):
        return self.R.ref_cache_drop(self.c, s)

    def fork(self, s):
        return self.R.ref_cache_fork(self.c, s)

    def truncate(self, s, n):
        return self.R.ref_cache_truncate(self.c, s, n)

    def insert(self, toks):
        return self.R.ref_radix_insert(self.c, _i32(toks), len(toks))

    def attach(self, node, s):
        return self.R.ref_radix_attach(self.c, node, s)

    def lookup(self, toks):
        node = C.c_uint64()
        n = self.R.ref_radix_lookup(self.c, _i32(toks), len(toks), C.byref(node))
        return node.value, n

    def reuse(self, toks, partial):
        n = C.c_size_t()
        s = self.R.ref_radix_reuse(self.c, _i32(toks), len(toks), partial, C.byref(n))
        return s, n.value

    def node_op(self, name, node):
        return getattr(self.R, "ref_radix_" + name)(self.c, node)

    def evict(self):
        return self.R.ref_radix_evict_one(self.c)

    def state(self, live):
        tables = {}
        for s in live:
            ids, gens = (C.c_size_t * 4096)(), (C.c_uint64 * 4096)()
            n = self.R.ref_cache_table(self.c, s, ids, gens)
            tables[s] = [(ids[i], gens[i]) for i in range(n)]
        return (self.R.ref_cache_available(self.c),
                [self.R.ref_cache_references(self.c, i) for i in range(self.blocks)],
                tables, self.R.ref_radix_size(self.c))

    def audit(self):
        return self.R.ref_cache_audit(self.c)


def _same(books, fn):
    out = [fn(b) for b in books]
    assert all(o == out[0] for o in out[1:]), out
    return out[0]


@pytest.mark.parametrize("blocks,tpb,vocab,seed", [(24, 2, 3, 0), (48, 4, 2, 1), (64, 3, 4, 2), (12, 4, 3, 3),
                                                   (96, 16, 2, 4)])
def test_prefix_trie_replays_reference(capi, ref_shim, blocks, tpb, vocab, seed):
    books = [Ours(capi, blocks, tpb), Ref(ref_shim, blocks, tpb)]
    rng = np.random.default_rng(seed)
    tokens = {}  # live sequence -> its token ids
    nodes = [0]  # node ids handed out so far (some later evicted)
    ops = ["new", "append", "append", "cache", "cache", "reuse", "reuse", "lookup", "pin", "unpin", "touch",
           "touch", "evict", "drop", "truncate", "fork"]
    for _ in range(500):
        op = str(rng.choice(ops))
        live = list(tokens)
        if op == "new" or not live:
            s = _same(books, lambda b: b.create())
            tokens[s] = []
            op = "append"
            live = [s]
        s = live[int(rng.integers(len(live)))]
        if op == "append":
            for _ in range(int(rng.integers(1, 7))):
                rc = _same(books, lambda b: b.append(s))
                if rc == 0:
                    tokens[s].append(int(rng.integers(vocab)))
        elif op == "cache" and tokens[s]:
            node = _same(books, lambda b: b.insert(tokens[s]))
            nodes.append(node)
            _same(books, lambda b: b.attach(node, s))
        elif op == "reuse":
            base = tokens[s] + [int(t) for t in rng.integers(vocab, size=int(rng.integers(0, 6)))]
            if base:
                partial = int(rng.integers(2))
                r, n = _same(books, lambda b: b.reuse(base, partial))
                if r:
                    tokens[r] = base[:n]
        elif op == "lookup":
            probe = [int(t) for t in rng.integers(vocab, size=int(rng.integers(0, 12)))]
            _same(books, lambda b: b.lookup(probe))
        elif op in ("pin", "unpin", "touch"):
            node = nodes[int(rng.integers(len(nodes)))] if rng.random() < 0.85 else int(rng.integers(0, 60))
            _same(books, lambda b: b.node_op(op, node))
        elif op == "evict":
            _same(books, lambda b: b.evict())
        elif op == "drop":
            _same(books, lambda b: b.drop(s))
            del tokens[s]
        elif op == "truncate":
            k = int(rng.integers(0, len(tokens[s]) + 1))
            _same(books, lambda b: b.truncate(s, k))
            tokens[s] = tokens[s][:k]
        elif op == "fork":
            f = _same(books, lambda b: b.fork(s))
            if f:
                tokens[f] = list(tokens[s])
        _same(books, lambda b: b.state(list(tokens)))
        assert all(b.audit() == 0 for b in books)
