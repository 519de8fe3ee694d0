"""PagedKVCache: a model's decode loop over per-layer page pools with one plan
per step (the attention of TransformerLayer::forward_with_cache,
crates/dendrite-core/src/model/layer.rs:374-416, with its grouped GQA),
against the oracle with the grouped map on the pools read back each step."""
import numpy as np
import pytest
import torch

import dendrite_b200 as dd
import oracle
from tests.helpers import assert_close, bf16_bits, bits_to_f32

pytestmark = pytest.mark.gpu

L, HQ, HKV, D, P = 2, 8, 2, 128, 64


def _bf16(x, dev):
    return torch.from_numpy(bf16_bits(x).view(np.int16).copy()).view(torch.bfloat16).to(dev)


def _pool_np(cache, layer, fmt):
    if fmt == "bf16":
        return cache.pools[layer].view(torch.int16).cpu().numpy().view(np.uint16)
    return oracle.dequantize(cache.pools[layer].cpu().numpy(), cache.scales[layer].cpu().numpy(), fmt,
                             out="bf16")


@pytest.mark.parametrize("fmt", ["bf16", "mxfp8"])
def test_decode_loop_over_paged_cache(cuda, fmt):
    rng = np.random.default_rng(12)
    cache = dd.PagedKVCache(L, P, HQ, HKV, D, kv_dtype=fmt, device=cuda)
    free = iter(range(P))
    prompt = [next(free), next(free)]                       # 32 shared prompt tokens
    tables = [prompt + [next(free)] for _ in range(3)]       # each sequence: own page for its tail
    lens = [32 + 5, 32 + 3, 32 + 9]                          # own prompt tokens after the shared ones
    # prompts: the shared 32 tokens once (sequence 0's table), then each tail
    for layer in range(L):
        q = rng.standard_normal((32, HQ, D)).astype(np.float32)
        k = rng.standard_normal((32, HKV, D)).astype(np.float32)
        v = rng.standard_normal((32, HKV, D)).astype(np.float32)
        out = cache.layer_prefill(layer, _bf16(q, cuda), _bf16(k, cuda), _bf16(v, cuda), tables[0], 0)
        # prompt token i sees tokens 0..i of the table (grouped GQA)
        torch.cuda.synchronize()
        ref, _ = oracle.decode_batch(bits_to_f32(bf16_bits(q)), _pool_np(cache, layer, fmt),
                                     np.arange(33, dtype=np.int32) * 3, np.tile(np.array(tables[0], np.uint32), 32),
                                     np.arange(1, 33, dtype=np.int32), HKV, gqa_grouped=True)
        assert_close(out.float().cpu().numpy(), bits_to_f32(bf16_bits(ref)), what="prompt")
        for b in range(3):
            n = lens[b] - 32
            qt = _bf16(rng.standard_normal((n, HQ, D)).astype(np.float32), cuda)
            kt = _bf16(rng.standard_normal((n, HKV, D)).astype(np.float32), cuda)
            vt = _bf16(rng.standard_normal((n, HKV, D)).astype(np.float32), cuda)
            cache.layer_prefill(layer, qt, kt, vt, tables[b], 32)
    torch.cuda.synchronize()
    advanced = []
    for step in range(20):
        if step == 10:   # fork sequence 1 (copy-on-write of its partial last page)
            src = tables[1][-1]
            dst = next(free)
            for layer in range(L):
                cache.pools[layer][dst] = cache.pools[layer][src]
                if cache.scales[layer] is not None:
                    cache.scales[layer][dst] = cache.scales[layer][src]
            tables.append(tables[1][:-1] + [dst])
            lens.append(lens[1])
        pos = np.array(lens)
        for b in range(len(tables)):
            if pos[b] % 16 == 0:
                tables[b].append(next(free))
        indptr = np.cumsum([0] + [len(t) for t in tables]).astype(np.int32)
        ids = np.concatenate(tables).astype(np.uint32)
        advanced.append(cache.begin_step(indptr, ids, pos))
        for layer in range(L):
            B = len(tables)
            q = rng.standard_normal((B, HQ, D)).astype(np.float32)
            k = rng.standard_normal((B, HKV, D)).astype(np.float32)
            v = rng.standard_normal((B, HKV, D)).astype(np.float32)
            out = cache.layer_step(layer, _bf16(q, cuda), _bf16(k, cuda), _bf16(v, cuda))
            torch.cuda.synchronize()
            ref, _ = oracle.decode_batch(bits_to_f32(bf16_bits(q)), _pool_np(cache, layer, fmt), indptr, ids,
                                         pos + 1, HKV, gqa_grouped=True)
            assert_close(out.float().cpu().numpy(), bits_to_f32(bf16_bits(ref)), what=f"step {step} layer {layer}")
        lens = [n + 1 for n in lens]
    assert not advanced[0] and all(advanced[1:10]) and not advanced[10] and all(advanced[11:])
