"""GPU parity of cascade / paged decode against the CPU oracle (C-ABI path)."""
import numpy as np
import pytest
import torch

import dendrite_b200 as dd
import oracle
from dendrite_b200 import _lib
from dendrite_b200 import workloads as wl
from tests.helpers import (F32_MAX_ABS, F32_MEAN_REL, FP8_MAX_ABS_CAP, FP8_MEAN_REL_CAP,
                           assert_close, bf16_bits, bits_to_f32, errors, random_pool)

pytestmark = pytest.mark.gpu


def to_dev_bf16(bits: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(dev)


def run_cascade(tb, pool_dev, q_dev, kv_dtype, scales=None, gqa=0, share=True, chunk=0, tc=True):
    cfg = dd.make_config(tb.num_qo_heads, tb.num_kv_heads, tb.head_dim, tb.num_pages,
                         kv_dtype=kv_dtype,
                         q_dtype=_lib.DTYPE_F32 if q_dev.dtype == torch.float32 else _lib.DTYPE_BF16,
                         gqa_map=gqa)
    plan = dd.CascadePlan(cfg, tb.indptr, tb.block_ids, tb.num_tokens, share_prefixes=share,
                          max_chunk_pages=chunk, use_tensor_cores=tc)
    plan.upload(q_dev.device)
    out, lse = dd.cascade_decode(cfg, plan, q_dev, pool_dev, scales)
    torch.cuda.synchronize()
    return out, lse


def oracle_ref(tb, pool_np, q_f32, gqa=0):
    return oracle.decode_batch(q_f32, pool_np, tb.indptr, tb.block_ids, tb.num_tokens,
                               tb.num_kv_heads, gqa_grouped=bool(gqa))


def test_golden_attention_f32(golden, cuda):
    g = golden["attention_small"]

    class TB:  # the golden batch as a tree batch
        num_qo_heads, num_kv_heads, head_dim = 8, 2, 64
        num_pages = g["pool"].shape[0]
        indptr, block_ids, num_tokens = g["indptr"], g["block_ids"], g["num_tokens"]

    out, lse = run_cascade(TB, torch.from_numpy(g["pool"]).to(cuda),
                           torch.from_numpy(g["q"]).to(cuda), _lib.DTYPE_F32)
    assert_close(out.cpu().numpy(), g["out"], F32_MAX_ABS, F32_MEAN_REL, "golden f32")
    l = lse.cpu().numpy()
    fin = np.isfinite(g["lse"])
    np.testing.assert_allclose(l[fin], g["lse"][fin], atol=1e-4)
    assert np.all(np.isneginf(l[3])) and torch.all(out[3] == 0)


CASES = [  # (Hq, Hkv, D, gqa)
    (8, 2, 128, 0), (32, 8, 128, 0), (32, 8, 128, 1), (8, 8, 128, 0), (32, 4, 64, 0),
    (16, 2, 64, 1), (64, 8, 128, 0), (128, 2, 128, 0),
]


@pytest.mark.parametrize("Hq,Hkv,D,gqa", CASES)
@pytest.mark.parametrize("share", [True, False])
def test_bf16_tree_vs_oracle(cuda, Hq, Hkv, D, gqa, share):
    seed = Hq * 7 + Hkv * 3 + D + gqa
    tb = wl.small_tree(seed, Hq=Hq, Hkv=Hkv, D=D, prefix=96, levels=((3, 16, 80), (2, 16, 48)),
                       leaves_per_node=2, suffix=(1, 70))
    rng = np.random.default_rng(seed)
    pool = bf16_bits(random_pool(rng, tb.num_pages, Hkv, D))
    q = bf16_bits(rng.standard_normal((tb.batch_size, Hq, D)).astype(np.float32))
    out, lse = run_cascade(tb, to_dev_bf16(pool, cuda), to_dev_bf16(q, cuda), _lib.DTYPE_BF16,
                           gqa=gqa, share=share)
    ref, ref_lse = oracle_ref(tb, pool, bits_to_f32(q), gqa)
    ref_b = bits_to_f32(bf16_bits(ref))  # the reference returns the query dtype
    assert_close(out.float().cpu().numpy(), ref_b, what=f"bf16 Hq{Hq} Hkv{Hkv} D{D}")
    np.testing.assert_allclose(lse.cpu().numpy(), ref_lse, atol=2e-3)


@pytest.mark.parametrize("chunk", [1, 2, 5])
def test_split_k_chunking(cuda, chunk):
    tb = wl.small_tree(11, Hq=32, Hkv=8, D=128, prefix=400, levels=((2, 64, 200),),
                       leaves_per_node=3, suffix=(1, 90))
    rng = np.random.default_rng(11)
    pool = bf16_bits(random_pool(rng, tb.num_pages, 8, 128))
    q = bf16_bits(rng.standard_normal((tb.batch_size, 32, 128)).astype(np.float32))
    out, _ = run_cascade(tb, to_dev_bf16(pool, cuda), to_dev_bf16(q, cuda), _lib.DTYPE_BF16,
                         chunk=chunk)
    ref, _ = oracle_ref(tb, pool, bits_to_f32(q))
    assert_close(out.float().cpu().numpy(), bits_to_f32(bf16_bits(ref)), what=f"chunk {chunk}")


def test_tinyllama_config_f32(cuda):
    """Config 1: Hq32/Hkv4/D64 f32, 4096-token prefix + 6 branches x 64."""
    tb = wl.tinyllama_tree()
    rng = np.random.default_rng(0xD3D1)
    pool = random_pool(rng, tb.num_pages, 4, 64)
    q = rng.standard_normal((6, 32, 64)).astype(np.float32)
    out, lse = run_cascade(tb, torch.from_numpy(pool).to(cuda), torch.from_numpy(q).to(cuda),
                           _lib.DTYPE_F32)
    ref, ref_lse = oracle_ref(tb, pool, q)
    assert_close(out.cpu().numpy(), ref, F32_MAX_ABS, F32_MEAN_REL, "tinyllama f32")
    np.testing.assert_allclose(lse.cpu().numpy(), ref_lse, atol=1e-4)


def test_tinyllama_config_bf16(cuda):
    tb = wl.tinyllama_tree()
    rng = np.random.default_rng(0xD3D2)
    pool = bf16_bits(random_pool(rng, tb.num_pages, 4, 64))
    q = bf16_bits(rng.standard_normal((6, 32, 64)).astype(np.float32))
    out, _ = run_cascade(tb, to_dev_bf16(pool, cuda), to_dev_bf16(q, cuda), _lib.DTYPE_BF16)
    ref, _ = oracle_ref(tb, pool, bits_to_f32(q))
    assert_close(out.float().cpu().numpy(), bits_to_f32(bf16_bits(ref)), what="tinyllama bf16")


@pytest.mark.parametrize("fmt", ["e4m3", "mxfp8"])
def test_fp8_tree_vs_oracle(cuda, fmt):
    tb = wl.small_tree(5, Hq=32, Hkv=8, D=128, prefix=128, levels=((3, 16, 96),),
                       leaves_per_node=3, suffix=(1, 60))
    rng = np.random.default_rng(5)
    pool = bf16_bits(random_pool(rng, tb.num_pages, 8, 128, outliers=1e-3))
    q = bf16_bits(rng.standard_normal((tb.batch_size, 32, 128)).astype(np.float32))
    codes, scales = dd.quantize_kv_pages(to_dev_bf16(pool, cuda), fmt)
    if fmt == "e4m3":
        oc, os_ = oracle.quantize_per_head(pool)
    else:
        oc, os_ = oracle.quantize_mx(pool)
    assert np.array_equal(codes.cpu().numpy(), oc)
    assert np.array_equal(scales.cpu().numpy(), os_)
    out, _ = run_cascade(tb, codes, to_dev_bf16(q, cuda),
                         _lib.DTYPE_E4M3 if fmt == "e4m3" else _lib.DTYPE_MXFP8, scales=scales)
    got = out.float().cpu().numpy()
    deq = oracle.dequantize(oc, os_, fmt, out="bf16")
    ref_fp8, _ = oracle_ref(tb, deq, bits_to_f32(q))
    assert_close(got, bits_to_f32(bf16_bits(ref_fp8)), what=f"{fmt} vs dequantised oracle")
    # Against the bf16-KV oracle: the bound is 1.25x the error of the oracle's
    # own FP8 path (FP8-dequant oracle vs bf16 oracle) on these inputs.
    ref_bf16, _ = oracle_ref(tb, pool, bits_to_f32(q))
    oma, omr = errors(ref_fp8, ref_bf16)
    assert oma <= FP8_MAX_ABS_CAP and omr <= FP8_MEAN_REL_CAP, (oma, omr)
    assert_close(got, ref_bf16, 1.25 * oma, 1.25 * omr, f"{fmt} vs bf16 oracle")


@pytest.mark.parametrize("kv", ["bf16", "f32", "e4m3"])
def test_decode_paged_device_tables(cuda, kv):
    rng = np.random.default_rng(21)
    Hq, Hkv, D, P = 32, 8, 128, 300
    ntok = np.array([1, 15, 16, 17, 200, 0, 1000, 33, 2047], dtype=np.int32)
    perm = rng.permutation(P).astype(np.uint32)
    tables, k = [], 0
    for n in ntok:
        nb = -(-int(n) // 16)
        tables.append(perm[k:k + nb])
        k += nb
    indptr = np.cumsum([0] + [len(t) for t in tables]).astype(np.int32)
    ids = np.concatenate(tables).astype(np.uint32)
    pool32 = random_pool(rng, P, Hkv, D)
    q32 = rng.standard_normal((len(ntok), Hq, D)).astype(np.float32)
    if kv == "f32":
        pool_np, pool_dev, qd, kvd, sc = pool32, torch.from_numpy(pool32).to(cuda), \
            torch.from_numpy(q32).to(cuda), _lib.DTYPE_F32, None
        qf = q32
    else:
        bits = bf16_bits(pool32)
        qb = bf16_bits(q32)
        qd, qf = to_dev_bf16(qb, cuda), bits_to_f32(qb)
        if kv == "bf16":
            pool_np, pool_dev, kvd, sc = bits, to_dev_bf16(bits, cuda), _lib.DTYPE_BF16, None
        else:
            pool_dev, sc = dd.quantize_kv_pages(to_dev_bf16(bits, cuda), "e4m3")
            pool_np = oracle.dequantize(pool_dev.cpu().numpy(), sc.cpu().numpy(), "e4m3")
            kvd = _lib.DTYPE_E4M3
    cfg = dd.make_config(Hq, Hkv, D, P, kv_dtype=kvd,
                         q_dtype=_lib.DTYPE_F32 if kv == "f32" else _lib.DTYPE_BF16)
    dev = lambda a: torch.from_numpy(a.astype(np.int32)).to(cuda)  # noqa: E731
    out, lse = dd.decode_paged(cfg, qd, pool_dev, dev(indptr), dev(ids), dev(ntok),
                               int(max(len(t) for t in tables)), kv_scales=sc)
    torch.cuda.synchronize()
    ref, ref_lse = oracle.decode_batch(qf, pool_np, indptr, ids, ntok, Hkv)
    got = out.float().cpu().numpy()
    if kv == "f32":
        assert_close(got, ref, F32_MAX_ABS, F32_MEAN_REL, "paged f32")
    else:
        assert_close(got, bits_to_f32(bf16_bits(ref)), what=f"paged {kv}")
    fin = np.isfinite(ref_lse)
    np.testing.assert_allclose(lse.cpu().numpy()[fin], ref_lse[fin], atol=2e-3)
    assert torch.all(out[5] == 0)


def test_decode_paged_reports_bad_page(cuda):
    Hq, Hkv, D, P = 8, 2, 128, 4
    cfg = dd.make_config(Hq, Hkv, D, P)
    pool = torch.randn(P, 2, Hkv, 16, D, device=cuda).to(torch.bfloat16)
    q = torch.randn(1, Hq, D, device=cuda).to(torch.bfloat16)
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device=cuda)  # noqa: E731
    ws = torch.empty(1 << 20, dtype=torch.uint8, device=cuda)
    dd.decode_paged(cfg, q, pool, i32([0, 2]), i32([1, 9]), i32([32]), 2, workspace=ws)
    code, aux = dd.workspace_status(ws)
    assert (code, aux) == (1, 9)
    dd.decode_paged(cfg, q, pool, i32([0, 2]), i32([1, 2]), i32([32]), 2, workspace=ws)
    assert dd.workspace_status(ws) == (0, 0)


def test_workspace_too_small(cuda):
    import ctypes as C

    tb = wl.small_tree(1)
    cfg = dd.make_config(tb.num_qo_heads, tb.num_kv_heads, tb.head_dim, tb.num_pages)
    plan = dd.CascadePlan(cfg, tb.indptr, tb.block_ids, tb.num_tokens)
    plan.upload(cuda)
    q = torch.zeros(tb.batch_size, tb.num_qo_heads, tb.head_dim, dtype=torch.bfloat16, device=cuda)
    pool = torch.zeros(tb.num_pages, 2, tb.num_kv_heads, 16, tb.head_dim, dtype=torch.bfloat16,
                       device=cuda)
    ws = torch.empty(plan.info().workspace_bytes - 256, dtype=torch.uint8, device=cuda)
    p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    rc = _lib.lib.dd_cascade_decode(C.byref(cfg), plan._h, p(q), p(pool), None, p(q), None, p(ws),
                                    ws.numel(), None)
    assert rc == _lib.DD_ERR_WORKSPACE


def test_merge_states_gpu_vs_oracle(cuda):
    rng = np.random.default_rng(3)
    o1, o2 = rng.standard_normal((2, 50, 128)).astype(np.float32)
    l1, l2 = (rng.standard_normal((2, 50)) * 4).astype(np.float32)
    l2[0] = -np.inf
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    o, l = dd.merge_states(t(o1), t(l1), t(o2), t(l2))
    ro, rl = oracle.merge_states(o1, l1, o2, l2)
    np.testing.assert_allclose(o.cpu().numpy(), ro, atol=1e-5)
    np.testing.assert_allclose(l.cpu().numpy(), rl, atol=1e-5)


def test_scatter_head_shards(cuda):
    Hq, Hkv, D, B, W = 64, 8, 128, 5, 4
    for gqa in (0, 1):
        cfg = dd.make_config(Hq, Hkv, D, 1, gqa_map=gqa)
        full = torch.randn(B, Hq, D, device=cuda).to(torch.bfloat16)
        g = Hq // Hkv
        shards = []
        for r in range(W):
            ks = range(r * Hkv // W, (r + 1) * Hkv // W)
            if gqa == 0:  # local head li = j * Hkv_r + (k - k0) -> global k + j * Hkv
                heads = [k + j * Hkv for j in range(g) for k in ks]
            else:
                heads = [k * g + j for k in ks for j in range(g)]
            shards.append(full[:, heads])
        gathered = torch.stack(shards).contiguous()
        out = torch.empty_like(full)
        dd.scatter_head_shards(cfg, W, gathered, out)
        torch.cuda.synchronize()
        assert torch.equal(out, full)
