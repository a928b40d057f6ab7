"""Failure detection on the GPU without a fault: the kernels' bounded waits.

Every pipeline wait inside the kernels gives up after a per-device time limit
(``cie_set_wait_limit``, 2 s by default). A wait that runs out records
CIE_DEV_TIMEOUT in the device status word, makes the kernel's other roles leave
their loops, lets the copies and MMAs already in flight land, releases tensor
memory and returns. These tests set the limit to 0, so that every wait that is
not satisfied at once runs out, on a small tcgen05 prefill and an HBM-bound
paged (TMA-fed) decode; they check the status bit, then restore the limit and
check that the next calls on the same context match the oracle.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests.golden.inputs import normal
from tests.helpers import assert_close_attn, to_np, to_torch

pytestmark = pytest.mark.gpu


def _prefill_inputs(cuda):
    import torch

    from kernels import build_rope_cache

    q = oracle.bf16_round(normal(901, (1, 8, 512, 128)))
    k = oracle.bf16_round(normal(902, (1, 2, 512, 128)))
    v = oracle.bf16_round(normal(903, (1, 2, 512, 128)))
    rope = build_rope_cache(512, 128, theta=500000.0, device=cuda)
    t = [to_torch(a, torch.bfloat16, cuda) for a in (q, k, v)]
    return (q, k, v), t, rope


def _paged_inputs(cuda):
    """A decode batch large enough to be HBM-bound (~270 MB of K/V), so that the
    warps' stage waits do find their tiles still in flight."""
    import torch

    from tests.test_paged_gpu import _device_pool

    lens = np.random.default_rng(906).integers(3000, 6000, size=32).tolist()
    kp, vp, tables = _device_pool(lens, 8, 64, 16, 904, cuda)
    q = normal(905, (32, 32, 1, 64))
    args = (to_torch(q, torch.bfloat16, cuda), kp, vp, torch.from_numpy(tables).to(cuda),
            torch.tensor(lens, dtype=torch.int32, device=cuda))
    return q, lens, tables, args


def test_wait_limit_runs_out_and_context_recovers(cuda):
    import torch

    from kernels import _lib
    from kernels.flash_attention import flash_attention, paged_attention
    from tests.test_paged_gpu import _check_sampled

    (q, k, v), tq, rope = _prefill_inputs(cuda)
    qd, lens, tables, pargs = _paged_inputs(cuda)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0

    prev = _lib.set_wait_limit(0)
    try:
        assert prev == _lib.DEFAULT_WAIT_LIMIT_NS
        flash_attention(*tq, causal=True, rope=rope)
        st_prefill = _lib.device_status(clear=True)   # synchronizes
        paged_attention(*pargs, True, split_tokens=256)
        st_paged = _lib.device_status(clear=True)
    finally:
        assert _lib.set_wait_limit(prev) == 0
    assert st_prefill & _lib.CIE_DEV_TIMEOUT, st_prefill
    assert st_paged & _lib.CIE_DEV_TIMEOUT, st_paged

    # same context, default limit: both kernels are correct again
    out = to_np(flash_attention(*tq, causal=True, rope=rope))
    c, s = oracle.build_rope_cache(512, 128, 500000.0)
    assert_close_attn(out, oracle.prefill_case_ref(q, k, v, c, s, causal=True), what="prefill")
    outd = to_np(paged_attention(*pargs, True, split_tokens=256))
    _check_sampled(outd, qd, pargs[1], pargs[2], tables, lens, [0, 13, 31], None, None, "paged")
    assert _lib.device_status(clear=True) == 0


def test_wait_limit_setter_roundtrip(cuda):
    from kernels import _lib

    prev = _lib.set_wait_limit(123456789)
    try:
        assert _lib.set_wait_limit(prev) == 123456789
    finally:
        _lib.set_wait_limit(_lib.DEFAULT_WAIT_LIMIT_NS)
    assert _lib.set_wait_limit(_lib.DEFAULT_WAIT_LIMIT_NS) == _lib.DEFAULT_WAIT_LIMIT_NS
