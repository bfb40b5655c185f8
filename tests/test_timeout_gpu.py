"""The bounded-wait (timeout) path of the tcgen05 decode kernel, exercised without faulting the GPU.

Every device-side wait of the decode kernel gives up after a bound (1 s by default). This test shortens
the bound to 2 ms and makes one V producer per CTA skip its loads (palu_set_wait_limit, a test hook), so
that a wait runs out on purpose. The kernel must then return on its own (no trap, no hang): the call's
status word reads 1, its merge writes NaN rather than numbers that look valid, the opt-in check of
``palu_sdpa_decode`` raises, and the next normal call on the same device and workspace is correct again.
"""
import pytest
import torch

import oracle
from oracle.metrics import MAX_REL, MEAN_REL, rowwise_rel_errors

pytestmark = pytest.mark.gpu


def _case(dev):
    g = torch.Generator().manual_seed(31)
    B, nkv, nh, S, r = 2, 8, 32, 1024, 64
    q, k, v, u, _ = oracle.seeded_decode_inputs(31, B, nkv, nh, S, r, r)
    pos = torch.tensor([S - 1, 500], dtype=torch.int32)
    cos, sin = oracle.cos_sin_tables(128, S, 500000.0, None)
    cos, sin = cos[:S].bfloat16().float(), sin[:S].bfloat16().float()
    return (q, k, v, u, pos, cos, sin), g


def test_expired_wait_reports_status_nan_and_recovers(cuda):
    from palu_b200 import _lib, fused
    (q, k, v, u, pos, cos, sin), _ = _case(cuda)
    S = k.shape[2]
    cs = fused.pack_cs_table(fused.cs_table(cos, sin, S).to(cuda, torch.bfloat16))
    d = _lib.dims(q.shape[1], q.shape[2], k.shape[1], k.shape[1], 64, 64, S)
    ws = _lib.new_workspace(d, cuda)
    args = (q[0].to(cuda, torch.bfloat16), k.to(cuda, torch.bfloat16), v.to(cuda, torch.bfloat16),
            u.to(cuda, torch.bfloat16), cs, pos.to(cuda))
    _lib.set_kernel(_lib.PALU_KERNEL_TC)
    try:
        assert _lib.kernel_for(d) == _lib.PALU_KERNEL_TC
        _lib.set_wait_limit(2_000_000, starve_v=True)
        out = fused.decode(*args, out_dtype=torch.float32, workspace=ws)
        torch.cuda.synchronize()
        assert _lib.read_status(ws) == 1, "the starved wait should have expired"
        assert torch.isnan(out).all(), "a failed call must not return numbers that look valid"
        # the opt-in check raises, as the reference op raises on a failed run
        with pytest.raises(RuntimeError, match="bounded device wait expired"):
            fused.decode(*args, out_dtype=torch.float32, workspace=ws, check_status=True)
        assert _lib.read_status(ws) == 0  # the check read (and cleared) the word
        _lib.set_wait_limit(0, starve_v=False)
        for _ in range(2):  # the device and the workspace are usable again
            out = fused.decode(*args, out_dtype=torch.float32, workspace=ws, check_status=True)
        torch.cuda.synchronize()
    finally:
        _lib.set_wait_limit(0, starve_v=False)
        _lib.set_kernel(_lib.PALU_KERNEL_AUTO)
    ref = oracle.reference_decode(q, k, u, v, pos, cos, sin, 128 ** -0.5)[0]
    rmx, rmn = rowwise_rel_errors(out.cpu(), ref)
    assert rmx <= MAX_REL and rmn <= MEAN_REL, (rmx, rmn)


def test_sticky_status_makes_every_later_call_nan_until_read(cuda):
    """The status word stays set until read: a later call on the same workspace writes NaN too."""
    from palu_b200 import _lib, fused
    (q, k, v, u, pos, cos, sin), _ = _case(cuda)
    S = k.shape[2]
    cs = fused.pack_cs_table(fused.cs_table(cos, sin, S).to(cuda, torch.bfloat16))
    d = _lib.dims(q.shape[1], q.shape[2], k.shape[1], k.shape[1], 64, 64, S)
    ws = _lib.new_workspace(d, cuda)
    args = (q[0].to(cuda, torch.bfloat16), k.to(cuda, torch.bfloat16), v.to(cuda, torch.bfloat16),
            u.to(cuda, torch.bfloat16), cs, pos.to(cuda))
    _lib.set_kernel(_lib.PALU_KERNEL_TC)
    try:
        _lib.set_wait_limit(2_000_000, starve_v=True)
        fused.decode(*args, out_dtype=torch.float32, workspace=ws)
        _lib.set_wait_limit(0, starve_v=False)
        out = fused.decode(*args, out_dtype=torch.float32, workspace=ws)
        torch.cuda.synchronize()
        assert torch.isnan(out).all()
        assert _lib.read_status(ws) == 1
        out = fused.decode(*args, out_dtype=torch.float32, workspace=ws)
        torch.cuda.synchronize()
        assert torch.isfinite(out).all() and _lib.read_status(ws) == 0
    finally:
        _lib.set_wait_limit(0, starve_v=False)
        _lib.set_kernel(_lib.PALU_KERNEL_AUTO)
