"""The decode layer (palu_b200/attention.py) against the reference's layer oracle.

Fixture ``layer_mlrd_llama3``: the reference's ``PaluRefAttention`` (reference.py:14-55; HF head order,
rotate-half RoPE, fp32) on a llama3-scaled M-LRD layer (4 query / 2 KV heads, r_k 32, r_v 64): a
24-token prefill, then two decode steps. The layer here runs q / K in Meta order with the interleaved
tables and V absorbed into ``wo_fused``, so agreement also checks those weight transforms.

Tolerance (written here): the latent caches and the op's q are bf16, as on the reference's device path
(its caches are bf16, attention.py:159-169). That rounding alone, with every op exact (the CPU models
below), moves this fixture's layer output by 2.1e-3 (prefill) to 3.1e-3 (decode) mean-abs relative, so
the bar is max-abs relative <= 2e-2 and mean-abs relative <= 5e-3 on the fp32 layer output.

The CPU tests run the same layer code with its two device ops replaced by CPU models (the oracle's
reference_decode and a cache write), which checks the layer algebra without a GPU; the GPU test runs
the CUDA library.
"""
import json

import pytest
import torch

import oracle
from oracle.metrics import rel_errors
from tests.conftest import load_golden

MAX_REL, MEAN_REL = 2e-2, 5e-3


def _layer_from_golden(device):
    from palu_b200.attention import PaluAttention
    from palu_b200.convert import LowRank
    d = load_golden("layer_mlrd_llama3")
    cfg = json.loads(bytes(d["cfg"]).decode())
    lr = LowRank(k_VT=d["k_VT"], k_U=d["k_U"], v_VT=d["v_VT"], v_U=d["v_U"])
    layer = PaluAttention(d["wq"], d["wo"], lr, cfg["num_attention_heads"], cfg["num_key_value_heads"],
                          max_batch=2, max_seq=64, rope_theta=cfg["rope_theta"], rope_scaling=cfg["rope_scaling"],
                          device=device)
    return layer, d


def _cpu_ops(layer):
    """CPU models of the two device ops: the cache write and reference_decode (fused.py:82-107)."""
    def append(new_k, new_v, pos, kc, vc):
        for b, p in enumerate(pos.tolist()):
            if 0 <= p < kc.shape[2]:
                kc[b, :, p] = new_k[b].to(kc.dtype)
                vc[b, :, p] = new_v[b].to(vc.dtype)

    def attend(q, kc, w_rot, cs_tab, vc, head_dim_v, pos, u_v=None, scale=None, out_dtype=None, rot_step=None,
               trans_mat=None):
        gs = w_rot.shape[1] // kc.shape[1]
        S = kc.shape[2]
        cs = cs_tab[0, 0, :S].float()
        cos, sin = cs[:, :128], cs[:, 128:]
        if rot_step is not None:  # Phase 2: chunk-relative angles (the op's rule, oracle.phase2_tables)
            cos, sin = oracle.phase2_tables(cos, sin)
        u_v_ = None if u_v is None else u_v[0].float()
        return oracle.reference_decode(q.float(), oracle.expand_groups(kc.float(), gs), w_rot[0, :, :, :128].float(),
                                       oracle.expand_groups(vc.float(), gs), pos.long(), cos, sin, scale, u_v=u_v_)
    layer.append_op, layer.attend_op = append, attend


def _check(got, want, what):
    mx, mn = rel_errors(got.float().cpu(), want.float())
    assert mx <= MAX_REL and mn <= MEAN_REL, f"{what}: max {mx:.3e} mean {mn:.3e}"


def _run(layer, d):
    y_pre = layer.forward_prefill(d["x_pre"])
    _check(y_pre, d["y_pre"], "prefill")
    P = d["x_pre"].shape[1]
    B = d["x_pre"].shape[0]
    for step, (x, y) in enumerate([(d["x_d1"], d["y_d1"]), (d["x_d2"], d["y_d2"])]):
        pos = torch.full((B,), P + step, dtype=torch.int32)
        out = layer.forward_decode(x[:, 0], pos)
        _check(out, y[:, 0], f"decode step {step}")


def test_layer_matches_reference_layer_on_cpu_models():
    layer, d = _layer_from_golden("cpu")
    _cpu_ops(layer)
    _run(layer, d)


def test_layer_reference_shapes_and_cpu_refusal():
    """[1, 1, B, dim] in / out like the reference's decode; the CUDA ops refuse CPU tensors loudly."""
    layer, d = _layer_from_golden("cpu")
    _cpu_ops(layer)
    layer.forward_prefill(d["x_pre"])
    out = layer.forward_decode(d["x_d1"][:, 0][None, None], torch.full((2,), 24, dtype=torch.int32))
    assert out.shape == (1, 1, 2, d["x_pre"].shape[-1])
    fresh, _ = _layer_from_golden("cpu")
    with pytest.raises(RuntimeError, match="CUDA"):
        fresh.forward_decode(d["x_d1"][:, 0], torch.full((2,), 0, dtype=torch.int32))


def test_layer_reference_call_surface():
    """The reference layer's call forms (attention.py:382, 585, 735-740): ``forward`` dispatches on
    ``mode``, ``rot_mats`` is the third positional argument of both forward methods (accepted, unused),
    ``page_table`` and ``kv_cache`` are keywords, and an external ``kv_cache`` is refused."""
    from palu_b200.attention import Mode
    a, d = _layer_from_golden("cpu")
    b, _ = _layer_from_golden("cpu")
    _cpu_ops(a)
    _cpu_ops(b)
    P, B = d["x_pre"].shape[1], d["x_pre"].shape[0]
    assert torch.equal(a.forward(d["x_pre"], None, None, 0, Mode.PREFILL), b.forward_prefill(d["x_pre"], None))
    pos = torch.full((B,), P, dtype=torch.int32)
    x = d["x_d1"][:, 0]
    want = b.forward_decode(x, pos, None, None, None)
    assert torch.equal(a.forward(x, pos, "ignored rot_mats", mode="decode"), want)
    with pytest.raises(RuntimeError, match="kv_cache"):
        a.forward_decode(x, pos, kv_cache=[object()])
    with pytest.raises(RuntimeError, match="chunked prefill"):
        a.forward_prefill(d["x_pre"], None, 0, chunk_start_idx=32)


@pytest.mark.gpu
def test_layer_matches_reference_layer_on_gpu(cuda):
    layer, d = _layer_from_golden("cuda")
    _run(layer, d)
    from palu_b200 import fused
    assert fused.workspace_status() == 0


def _glrd_case(seed=3, P=20):
    """A G-LRD layer (2 groups of 2 KV heads, ranks 48 / 96) and the oracle layer (reference.py:14-55) on it:
    a P-token prefill and one decode step."""
    from palu_b200.convert import LowRank
    g = torch.Generator().manual_seed(seed)
    nh, nkv, gs, hd, r_k, r_v = 8, 4, 2, 128, 48, 96
    dim = nh * hd
    bf = lambda t: t.to(torch.bfloat16).float()
    w = {"q": bf(torch.randn(dim, dim, generator=g) / dim ** 0.5), "o": bf(torch.randn(dim, dim, generator=g) / dim ** 0.5)}
    kvt = bf(torch.randn(nkv // gs, r_k, dim, generator=g) / dim ** 0.5).repeat_interleave(gs, 0)
    vvt = bf(torch.randn(nkv // gs, r_v, dim, generator=g) / dim ** 0.5).repeat_interleave(gs, 0)
    lr = LowRank(k_VT=kvt, k_U=bf(torch.randn(nkv, hd, r_k, generator=g) / r_k ** 0.5), v_VT=vvt,
                 v_U=bf(torch.randn(nkv, hd, r_v, generator=g) / r_v ** 0.5), group_size=gs)
    cfg = dict(hidden_size=dim, num_attention_heads=nh, num_key_value_heads=nkv, num_hidden_layers=1,
               intermediate_size=128, vocab_size=256, max_position_embeddings=131072, rope_theta=500000.0,
               rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                             "original_max_position_embeddings": 8192})
    ref = oracle.PaluRefAttention(cfg, w, lr)
    B = 2
    x_pre, x_d = bf(torch.randn(B, P, dim, generator=g)), bf(torch.randn(B, 1, dim, generator=g))
    return cfg, w, lr, x_pre, x_d, ref.forward(x_pre, 0), ref.forward(x_d, P)


def _glrd_layer(device, P=20, max_seq=48, cs_recurrence=False):
    from palu_b200.attention import PaluAttention
    cfg, w, lr, x_pre, x_d, y_pre, y_d = _glrd_case(P=P)
    layer = PaluAttention(w["q"], w["o"], lr, cfg["num_attention_heads"], cfg["num_key_value_heads"], max_batch=2,
                          max_seq=max_seq, rope_scaling=cfg["rope_scaling"], device=device,
                          cs_recurrence=cs_recurrence)
    return layer, x_pre, x_d, y_pre, y_d


def test_glrd_layer_matches_oracle_layer_on_cpu_models():
    layer, x_pre, x_d, y_pre, y_d = _glrd_layer("cpu")
    _cpu_ops(layer)
    _check(layer.forward_prefill(x_pre), y_pre, "G-LRD prefill")
    _check(layer.forward_decode(x_d[:, 0], torch.full((2,), x_pre.shape[1], dtype=torch.int32)), y_d[:, 0], "G-LRD decode")


def test_glrd_layer_phase2_matches_oracle_layer_on_cpu_models():
    """cs_recurrence=True (the reference's Phase 2): a 300-token prefill, so the decode step's keys span
    three 128-position chunks, still within the layer bar against the oracle layer's exact RoPE."""
    layer, x_pre, x_d, y_pre, y_d = _glrd_layer("cpu", P=300, max_seq=320, cs_recurrence=True)
    _cpu_ops(layer)
    _check(layer.forward_prefill(x_pre), y_pre, "G-LRD prefill")
    _check(layer.forward_decode(x_d[:, 0], torch.full((2,), x_pre.shape[1], dtype=torch.int32)), y_d[:, 0],
           "G-LRD Phase 2 decode")


@pytest.mark.gpu
def test_glrd_layer_phase2_matches_oracle_layer_on_gpu(cuda):
    layer, x_pre, x_d, y_pre, y_d = _glrd_layer("cuda", P=300, max_seq=320, cs_recurrence=True)
    _check(layer.forward_prefill(x_pre), y_pre, "G-LRD prefill")
    _check(layer.forward_decode(x_d[:, 0], torch.full((2,), x_pre.shape[1], dtype=torch.int32)), y_d[:, 0],
           "G-LRD Phase 2 decode")


@pytest.mark.gpu
def test_glrd_layer_matches_oracle_layer_on_gpu(cuda):
    layer, x_pre, x_d, y_pre, y_d = _glrd_layer("cuda")
    _check(layer.forward_prefill(x_pre), y_pre, "G-LRD prefill")
    _check(layer.forward_decode(x_d[:, 0], torch.full((2,), x_pre.shape[1], dtype=torch.int32)), y_d[:, 0], "G-LRD decode")


@pytest.mark.gpu
@pytest.mark.parametrize("latent_dtype,bar", [("f8", 0.99), ("f4", 0.95)])
def test_layer_with_low_bit_latent_caches(cuda, latent_dtype, bar):
    """The layer with the reference's low-bit latent-cache option (latent_dtype; bfp8 / bfp4 on the reference,
    e4m3 / e2m1 with power-of-two scales here): prefill and two decode steps against the same layer on bf16
    caches, PCC >= 0.99 (fp8) and >= 0.95 (fp4, the reference's bar for bfp4 latents)."""
    from palu_b200.attention import PaluAttention
    from palu_b200.convert import LowRank
    g = torch.Generator().manual_seed(41)
    nh, nkv, hd, r_k, r_v = 8, 4, 128, 64, 128
    dim = nh * hd
    bf = lambda t: t.to(torch.bfloat16).float()
    wq, wo = bf(torch.randn(dim, dim, generator=g) / dim ** 0.5), bf(torch.randn(dim, dim, generator=g) / dim ** 0.5)
    lr = LowRank(k_VT=bf(torch.randn(nkv, r_k, dim, generator=g) / dim ** 0.5),
                 k_U=bf(torch.randn(nkv, hd, r_k, generator=g) / r_k ** 0.5),
                 v_VT=bf(torch.randn(nkv, r_v, dim, generator=g) / dim ** 0.5),
                 v_U=bf(torch.randn(nkv, hd, r_v, generator=g) / r_v ** 0.5))
    layers = [PaluAttention(wq, wo, lr, nh, nkv, max_batch=2, max_seq=96, device="cuda", latent_dtype=ld)
              for ld in ("bf16", latent_dtype)]
    B, P = 2, 40
    x_pre = bf(torch.randn(B, P, dim, generator=g))
    xs = [bf(torch.randn(B, dim, generator=g)) for _ in range(2)]
    outs = []
    for layer in layers:
        o = [layer.forward_prefill(x_pre).cpu()]
        for i, x in enumerate(xs):
            o.append(layer.forward_decode(x, torch.full((B,), P + i, dtype=torch.int32)).cpu())
        outs.append(o)
    for a, b in zip(*outs):
        a, b = a.double().flatten(), b.double().flatten()
        a, b = a - a.mean(), b - b.mean()
        assert float((a @ b) / (a.norm() * b.norm())) >= bar
