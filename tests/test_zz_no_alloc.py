"""palu_decode_attn_static (the entry point that allocates nothing) against palu_decode_attn.

The static variant serves callers that cannot allocate a workspace: a plugin that only holds the tensors
its framework passes in, or a decode loop that must not call cudaMalloc per step. Both entry points are
called through the C ABI with the same arguments; the static variant keeps its partial results in the
library's static device scratch instead of a caller workspace. Two calls in a row with
different queries and positions must each match the workspace entry point within the parity bar the
other GPU tests use (max-abs relative <= 2e-2, mean-abs relative <= 1e-3), so stale scratch contents
from the first call cannot leak into the second. This file is collected last so that it runs both
alone and after the rest of the suite.
"""
import ctypes

import pytest
import torch

import oracle
from oracle.metrics import MAX_REL, MEAN_REL, rel_errors

pytestmark = pytest.mark.gpu

THETA = 500000.0


def _case(g, dev, B, nkv, n_lat, S, r_k, r_v, grouped):
    bf = torch.bfloat16
    k_lat = torch.randn(B, n_lat, S, r_k, generator=g).to(dev, bf)
    v_lat = torch.randn(B, n_lat, S, r_v, generator=g).to(dev, bf)
    u_k = (torch.randn(nkv, r_k, 128, generator=g) / r_k ** 0.5).to(dev, bf)
    u_v = (torch.randn(nkv, r_v, 128, generator=g) / r_v ** 0.5).to(dev, bf) if grouped else None
    cos, sin = oracle.cos_sin_tables(128, S, THETA, None)
    return k_lat, v_lat, u_k, u_v, cos[:S], sin[:S]


def _call(lib, static, q, k_lat, v_lat, u_k, u_v, cs_pairs, pos, out, d, ws):
    from palu_b200 import _lib
    stream = _lib.stream_handle(q.device)
    common = (q.data_ptr(), k_lat.data_ptr(), v_lat.data_ptr(), u_k.data_ptr(), 128, _lib.ptr(u_v),
              cs_pairs.data_ptr(), pos.data_ptr(), out.data_ptr(), _lib.PALU_F32)
    if static:
        return lib.palu_decode_attn_static(*common, ctypes.byref(d), 128 ** -0.5, stream)
    return lib.palu_decode_attn(*common, ws.data_ptr(), ws.numel(), ctypes.byref(d), 128 ** -0.5, stream)


@pytest.fixture(params=["tc", "mma"])
def kernel_family(request, cuda):
    """Both kernel families keep their partials in the static scratch; the choice is restored afterwards."""
    from palu_b200 import _lib
    _lib.set_kernel(_lib.PALU_KERNEL_TC if request.param == "tc" else _lib.PALU_KERNEL_MMA)
    try:
        yield request.param
    finally:
        _lib.set_kernel(_lib.PALU_KERNEL_AUTO)


# (B, KV heads, latent heads, S, r_k, r_v): M-LRD with absorbed V, and grouped latents with V rebuilt per head
CASES = [(8, 8, 8, 2048, 64, 64), (4, 8, 2, 1500, 128, 128)]


@pytest.mark.parametrize("case", CASES, ids=["mlrd", "grouped_uv"])
def test_static_scratch_matches_workspace_entry_point_twice(cuda, kernel_family, case):
    from palu_b200 import _lib, fused
    lib = _lib.load()
    g = torch.Generator().manual_seed(7)
    B, nkv, n_lat, S, r_k, r_v = case
    nh = 4 * nkv
    grouped = n_lat != nkv
    k_lat, v_lat, u_k, u_v, cos, sin = _case(g, cuda, B, nkv, n_lat, S, r_k, r_v, grouped)
    cs_pairs = fused.pack_cs_table(fused.cs_table(cos, sin, S).to(cuda, torch.bfloat16))
    d = _lib.dims(B, nh, nkv, n_lat, r_k, r_v, S)
    ws = _lib.new_workspace(d, cuda)
    width = 128 if grouped else r_v
    for call in range(2):
        q = torch.randn(B, nh, 128, generator=g).to(cuda, torch.bfloat16)
        pos = torch.randint(0, S, (B,), generator=g, dtype=torch.int32)
        pos[call] = S - 1
        pos = pos.to(cuda)
        want = torch.full((B, nh, width), float("nan"), device=cuda)
        got = torch.full((B, nh, width), float("nan"), device=cuda)
        _lib.check(_call(lib, False, q, k_lat, v_lat, u_k, u_v, cs_pairs, pos, want, d, ws))
        _lib.check(_call(lib, True, q, k_lat, v_lat, u_k, u_v, cs_pairs, pos, got, d, None))
        torch.cuda.synchronize()
        assert _lib.read_status(ws) == 0, "a bounded device wait expired (workspace call)"
        assert _lib.read_status(None) == 0, "a bounded device wait expired (static scratch)"
        assert torch.isfinite(got).all(), f"call {call}: output not fully written"
        mx, mn = rel_errors(got.cpu(), want.cpu())
        assert mx <= MAX_REL and mn <= MEAN_REL, f"call {call}: max {mx:.3e} mean {mn:.3e}"


def test_static_scratch_rejects_oversize_shapes(cuda):
    from palu_b200 import _lib
    lib = _lib.load()
    # 256 CTAs per KV head: partial records for either kernel family need more than the 8 MiB scratch,
    # so the call is refused before any pointer is used (the pointers here are dummies).
    d = _lib.dims(64, 32, 8, 8, 128, 128, 8192, splits=256)
    assert _lib.workspace_bytes(d) > 8 << 20
    st = lib.palu_decode_attn_static(1, 1, 1, 1, 128, None, 16, 1, 1, _lib.PALU_BF16, ctypes.byref(d), 1.0, None)
    assert st == _lib.PALU_ERR_WORKSPACE
    assert "static scratch" in lib.palu_last_error().decode()
