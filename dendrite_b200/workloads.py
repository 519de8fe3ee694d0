"""Seeded synthetic reasoning trees with copy-on-write block tables.

The block tables are produced the way Dendrite's TreeState produces them:
fork clones the parent's table and bumps block refcounts
(crates/dendrite-core/src/tree/state.rs:49-84); appending a token allocates a
block from the pool's FIFO free list when the last block is full
(state.rs:87-113, BlockTable::needs_new_block
crates/dendrite-core/src/cache/block_table.rs:88-94) and copy-on-writes a
shared last block (crates/dendrite-core/src/cache/pool.rs:76-97). The free list
starts as a seeded permutation of the pool, so physical pages are
non-contiguous. Internal (forked) nodes are 16-token aligned, as the reference's
CoW does not copy a partial block's data (pool.rs:88-91).

The shapes are the benchmark configurations of this path; there is no public
dataset behind them. KV values are N(0, 1) from a seed.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field

import numpy as np

PAGE = 16


class BlockPool:
    """Refcounted FIFO block pool (mirror of cache/pool.rs:40-97)."""

    def __init__(self, num_blocks: int, rng: np.random.Generator | None = None):
        order = np.arange(num_blocks, dtype=np.uint32)
        if rng is not None:
            rng.shuffle(order)
        self.free = deque(order.tolist())
        self.ref = np.zeros(num_blocks, dtype=np.int32)
        self.num_blocks = num_blocks

    def allocate(self) -> int:
        if not self.free:
            raise MemoryError("no free blocks")  # DendriteError::OutOfMemory (pool.rs:40-45)
        b = self.free.popleft()
        self.ref[b] = 1
        return b

    def share(self, b: int) -> None:
        self.ref[b] += 1

    def release(self, b: int) -> None:
        self.ref[b] -= 1
        if self.ref[b] == 0:
            self.free.append(b)

    def copy_on_write(self, b: int) -> int:
        if self.ref[b] <= 1:
            return b
        nb = self.allocate()
        self.release(b)
        return nb


@dataclass
class Sequence:
    """A tree node's sequence: its BlockTable (block ids + num_tokens)."""

    blocks: list = field(default_factory=list)
    num_tokens: int = 0


class TreeBuilder:
    """Mirror of TreeState::{fork, append_token} over a BlockPool."""

    def __init__(self, pool: BlockPool):
        self.pool = pool

    def root(self, tokens: int) -> Sequence:
        s = Sequence()
        self.append(s, tokens)
        return s

    def fork(self, parent: Sequence) -> Sequence:
        for b in parent.blocks:
            self.pool.share(b)
        return Sequence(list(parent.blocks), parent.num_tokens)

    def append(self, s: Sequence, n: int) -> None:
        if n <= 0:
            return
        if s.blocks and s.num_tokens % PAGE:
            s.blocks[-1] = self.pool.copy_on_write(s.blocks[-1])
        have = len(s.blocks) * PAGE
        while have < s.num_tokens + n:
            s.blocks.append(self.pool.allocate())
            have += PAGE
        s.num_tokens += n


@dataclass
class TreeBatch:
    """A decode batch: one query per leaf, with CSR block tables."""

    name: str
    num_qo_heads: int
    num_kv_heads: int
    head_dim: int
    num_pages: int
    indptr: np.ndarray      # int32 [B+1]
    block_ids: np.ndarray   # uint32
    num_tokens: np.ndarray  # int32 [B]
    unique_tokens: int      # KV tokens of the tree, each shared node counted once

    @property
    def batch_size(self) -> int:
        return len(self.num_tokens)

    def tables(self) -> list[list[int]]:
        return [self.block_ids[self.indptr[i]:self.indptr[i + 1]].tolist()
                for i in range(self.batch_size)]


def _csr(leaves: list[Sequence]):
    indptr = np.zeros(len(leaves) + 1, dtype=np.int32)
    for i, s in enumerate(leaves):
        indptr[i + 1] = indptr[i] + len(s.blocks)
    ids = np.fromiter((b for s in leaves for b in s.blocks), dtype=np.uint32, count=int(indptr[-1]))
    ntok = np.array([s.num_tokens for s in leaves], dtype=np.int32)
    return indptr, ids, ntok


def build_tree(name: str, Hq: int, Hkv: int, D: int, prefix: int, levels: list[tuple[int, int, int]],
               leaves_per_node: int, suffix: tuple[int, int], seed: int,
               num_trees: int = 1) -> TreeBatch:
    """Generic tree: a root prefix, then `levels` of (fan-out, min, max) tokens
    (16-aligned, internal), then `leaves_per_node` leaves per last-level node
    with a private suffix of U[suffix] tokens."""
    rng = np.random.default_rng(seed)
    shape_rng = np.random.default_rng(seed + 1)
    # Plan the token counts first to size the pool exactly.
    plans = []
    pages = 0
    for _ in range(num_trees):
        tree = {"prefix": prefix, "levels": [], "leaves": []}
        pages += -(-prefix // PAGE)
        count = 1
        for fan, lo, hi in levels:
            count *= fan
            lens = shape_rng.integers(lo // PAGE, hi // PAGE + 1, size=count) * PAGE
            tree["levels"].append(lens)
            pages += int(sum(-(-int(x) // PAGE) for x in lens))
        count *= leaves_per_node
        sl = shape_rng.integers(suffix[0], suffix[1] + 1, size=count)
        tree["leaves"] = sl
        pages += int(sum(-(-int(x) // PAGE) for x in sl)) + count  # + CoW slack
        plans.append(tree)
    pool = BlockPool(pages, rng)
    tb = TreeBuilder(pool)
    leaves: list[Sequence] = []
    unique = 0
    for tree in plans:
        frontier = [tb.root(tree["prefix"])]
        unique += tree["prefix"]
        for (fan, _, _), lens in zip(levels, tree["levels"]):
            nxt = []
            k = 0
            for parent in frontier:
                for _ in range(fan):
                    c = tb.fork(parent)
                    tb.append(c, int(lens[k]))
                    unique += int(lens[k])
                    k += 1
                    nxt.append(c)
            frontier = nxt
        k = 0
        for parent in frontier:
            for _ in range(leaves_per_node):
                c = tb.fork(parent)
                tb.append(c, int(tree["leaves"][k]))
                unique += int(tree["leaves"][k])
                k += 1
                leaves.append(c)
    indptr, ids, ntok = _csr(leaves)
    return TreeBatch(name, Hq, Hkv, D, pages, indptr, ids, ntok, unique)


# ---------------------------------------------------------------- configs
def tinyllama_tree(seed: int = 0xD3D1) -> TreeBatch:
    """Config 1: Hq32/Hkv4/D64, one 4096-token prefix, 6 branches x 64 tokens."""
    return build_tree("tinyllama-4096+6x64", 32, 4, 64, 4096, [], 6, (64, 64), seed)


def mcts_llama3_8b(seed: int = 0xD3D1, leaves: int = 512) -> TreeBatch:
    """Config 3: Hq32/Hkv8/D128; root 8192; depths 1-3 fan-out 8/4/4 with
    16-aligned nodes of 128-1024 tokens; 4 leaves per depth-3 node (512
    leaves) with U[16, 256]-token suffixes."""
    assert leaves % 128 == 0
    return build_tree("mcts-llama3-8b-512leaf", 32, 8, 128, 8192,
                      [(8, 128, 1024), (4, 128, 1024), (4, 128, 1024)], leaves // 128,
                      (16, 256), seed)


def llama3_70b_forest(num_trees: int = 64, seed: int = 0xD3D1) -> TreeBatch:
    """Config 5a: Hq64/Hkv8/D128; trees of a 32768-token prefix and 64
    branches x 256 tokens."""
    return build_tree("llama3-70b-forest", 64, 8, 128, 32768, [], 64, (256, 256), seed,
                      num_trees=num_trees)


def llama3_70b_long(seed: int = 0xD3D1, branches: int = 256) -> TreeBatch:
    """Config 5b: Hq64/Hkv8/D128; one 131072-token prefix, 256 branches x 256."""
    return build_tree("llama3-70b-131k", 64, 8, 128, 131072, [], branches, (256, 256), seed)


@dataclass
class PrefillBatch:
    """Chunked prefill of branch suffixes: sequence s holds prefix_len[s] +
    num_new[s] tokens in its CSR block table; its num_new[s] new tokens are
    the queries (sequence-major)."""

    name: str
    num_qo_heads: int
    num_kv_heads: int
    head_dim: int
    num_pages: int
    indptr: np.ndarray      # int32 [S+1]
    block_ids: np.ndarray   # uint32
    prefix_len: np.ndarray  # int32 [S]
    num_new: np.ndarray     # int32 [S]
    unique_tokens: int      # KV tokens, shared prefix pages counted once

    def nested(self) -> TreeBatch:
        """The same work as a decode batch: new token i of sequence s is a
        query over the sequence's table with prefix_len[s] + i + 1 tokens."""
        ptr, ids, ntok = [0], [], []
        for s in range(len(self.num_new)):
            tbl = self.block_ids[self.indptr[s]:self.indptr[s + 1]]
            for i in range(int(self.num_new[s])):
                ids.append(tbl)
                ptr.append(ptr[-1] + len(tbl))
                ntok.append(int(self.prefix_len[s]) + i + 1)
        return TreeBatch(self.name + "-nested", self.num_qo_heads, self.num_kv_heads, self.head_dim,
                         self.num_pages, np.array(ptr, np.int32),
                         np.concatenate(ids).astype(np.uint32) if ids else np.zeros(0, np.uint32),
                         np.array(ntok, np.int32), self.unique_tokens)


def prefill_branches_8b(seed: int = 0xD3D1, prefix: int = 8192, branches: int = 16,
                        new: int = 64) -> PrefillBatch:
    """Llama-3-8B heads (Hq32/Hkv8/D128): one shared prefix, then `branches`
    forks that each prefill `new` tokens (TreeState fork + append semantics:
    a partial last prefix page is copied on write)."""
    rng = np.random.default_rng(seed)
    pages = -(-prefix // PAGE) + branches * (-(-new // PAGE) + 1)
    pool = BlockPool(pages, rng)
    tb = TreeBuilder(pool)
    root = tb.root(prefix)
    seqs = []
    for _ in range(branches):
        c = tb.fork(root)
        tb.append(c, new)
        seqs.append(c)
    indptr, ids, _ = _csr(seqs)
    return PrefillBatch(f"prefill-llama3-8b-{prefix}+{branches}x{new}", 32, 8, 128, pages, indptr, ids,
                        np.full(branches, prefix, np.int32), np.full(branches, new, np.int32),
                        prefix + branches * new)


def small_tree(seed: int, Hq: int = 8, Hkv: int = 2, D: int = 128, prefix: int = 64,
               levels=((2, 16, 48),), leaves_per_node: int = 3, suffix=(1, 40)) -> TreeBatch:
    """Small random trees for parity tests."""
    return build_tree("small", Hq, Hkv, D, prefix, list(levels), leaves_per_node, tuple(suffix),
                      seed)


def effective_bytes(tb: TreeBatch, kv_bytes_per_elem: float, q_bytes: int = 2, out_bytes: int = 2,
                    scale_bytes_per_token_head: float = 0.0) -> int:
    """Algorithmic HBM bytes of one cascade decode step: every unique KV
    token of the tree once (K and V, all KV heads), its scale bytes, plus the
    queries read and outputs written."""
    H, D = tb.num_kv_heads, tb.head_dim
    kv = tb.unique_tokens * 2 * H * (D * kv_bytes_per_elem + scale_bytes_per_token_head)
    qo = tb.batch_size * tb.num_qo_heads * D * (q_bytes + out_bytes)
    return int(kv + qo)
