"""Failure detection without a GPU fault: a kernel's bounded mbarrier wait is
made to run out (a barrier nothing arrives on, 1 ms limit); the kernel gives
up and returns, the host reads the timeout from the workspace status, and the
context stays usable for the next decode."""
import numpy as np
import pytest
import torch

import dendrite_b200 as dd
import oracle
from dendrite_b200 import workloads as wl
from tests.helpers import assert_close, bf16_bits, bits_to_f32, random_pool

pytestmark = pytest.mark.gpu


def test_wait_timeout_is_reported_and_context_survives(cuda):
    ws = torch.zeros(1 << 20, dtype=torch.uint8, device=cuda)
    dd.selftest_wait(ws, 1_000_000)
    assert dd.workspace_status(ws) == (2, 0)       # status 2: a bounded wait timed out
    # the same context and workspace decode normally afterwards
    tb = wl.small_tree(4, Hq=8, Hkv=2, D=128)
    rng = np.random.default_rng(4)
    pool = bf16_bits(random_pool(rng, tb.num_pages, 2, 128))
    q = bf16_bits(rng.standard_normal((tb.batch_size, 8, 128)).astype(np.float32))
    dev = lambda b: torch.from_numpy(b.view(np.int16).copy()).view(torch.bfloat16).to(cuda)  # noqa: E731
    cfg = dd.make_config(8, 2, 128, tb.num_pages)
    plan = dd.CascadePlan(cfg, tb.indptr, tb.block_ids, tb.num_tokens)
    plan.upload(cuda)
    out, _ = dd.cascade_decode(cfg, plan, dev(q), dev(pool), workspace=ws)
    torch.cuda.synchronize()
    assert dd.workspace_status(ws) == (0, 0)
    ref, _ = oracle.decode_batch(bits_to_f32(q), pool, tb.indptr, tb.block_ids, tb.num_tokens, 2)
    assert_close(out.float().cpu().numpy(), bits_to_f32(bf16_bits(ref)), what="after timeout")


def test_selftest_rejects_bad_limits(cuda):
    ws = torch.zeros(256, dtype=torch.uint8, device=cuda)
    with pytest.raises(dd.InvalidArgument):
        dd.selftest_wait(ws, 0)
    with pytest.raises(dd.InvalidArgument):
        dd.selftest_wait(ws, 10_000_000_000)
