"""The oracle (oracle/) pinned against the reference's own outputs (tests/golden, produced by the
reference's Python code) and against the published pieces it restates. CPU only."""
import json
import math

import pytest
import torch

import oracle
from tests.conftest import load_golden

HD = 128
LLAMA3 = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
          "original_max_position_embeddings": 8192}


@pytest.mark.parametrize("name", ["decode_mlrd_r64", "decode_mlrd_rk32_rv128", "decode_identity_r128",
                                  "decode_glrd_gs4", "decode_mlrd_plain_rope"])
def test_oracle_reproduces_reference_decode_golden(name):
    d = load_golden(name)
    gs = int(d["group_size"])
    k = oracle.expand_groups(d["k_lat"], gs)
    v = oracle.expand_groups(d["v_lat"], gs)
    out = oracle.reference_decode(d["q"], k, d["u_k"], v, d["cur_pos"], d["cos"], d["sin"], float(d["scale"]),
                                  u_v=d.get("u_v"))
    torch.testing.assert_close(out, d["out"], atol=1e-6, rtol=1e-6)
    streamed = oracle.reference_decode_streamed(d["q"], d["k_lat"], d["u_k"], d["v_lat"], d["cur_pos"], d["cos"],
                                                d["sin"], float(d["scale"]), u_v=d.get("u_v"), group_size=gs)
    torch.testing.assert_close(streamed, d["out"], atol=2e-5, rtol=1e-4)


def test_layer_oracle_reproduces_reference_attention_golden():
    d = load_golden("layer_mlrd_llama3")
    cfg = json.loads(bytes(d["cfg"]).decode())

    class LR:
        k_VT, k_U, v_VT, v_U = d["k_VT"], d["k_U"], d["v_VT"], d["v_U"]

    ref = oracle.PaluRefAttention(cfg, {"q": d["wq"], "o": d["wo"]}, LR)
    torch.testing.assert_close(ref.forward(d["x_pre"], 0), d["y_pre"], atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(ref.forward(d["x_d1"], 24), d["y_d1"], atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(ref.forward(d["x_d2"], 25), d["y_d2"], atol=1e-5, rtol=1e-5)


def test_tables_equal_hf_llama_rotary_bit_for_bit():
    """The restated compute_gather_cos_sin frequencies == HF LlamaRotaryEmbedding (reference.py:22)."""
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding
    for rs in (None, LLAMA3):
        cfg = LlamaConfig(hidden_size=4096, num_attention_heads=32, num_key_value_heads=8, rope_theta=500000.0,
                          rope_scaling=dict(rs) if rs else None, max_position_embeddings=131072)
        rot = LlamaRotaryEmbedding(config=cfg)
        cos, sin = oracle.cos_sin_tables(HD, 2048, 500000.0, rs)
        c_hf, s_hf = rot(torch.zeros(1, 1, 8), torch.arange(cos.shape[0])[None])
        assert torch.equal(c_hf[0, :, :64], cos[:, 0::2]) and torch.equal(s_hf[0, :, :64], sin[:, 0::2])


def test_transformation_matrix_is_the_pair_rotation():  # restates tests/test_fused.py:8-17
    T = oracle.rope_transformation_matrix(HD)
    x = torch.randn(3, HD)
    r = x @ T
    torch.testing.assert_close(r[:, 0::2], -x[:, 1::2])
    torch.testing.assert_close(r[:, 1::2], x[:, 0::2])
    t = oracle.trans_mat_tile()
    assert t.shape == (1, 1, 32, 32) and torch.equal(t[0, 0], T[:32, :32])


def test_chunk_size_rule():  # tests/test_fused.py:28-30
    assert [oracle.chunk_size(s) for s in (96, 256, 1024, 4096, 8192, 8192 + 32)] == [32, 256, 512, 512, 512, 32]


def test_tables_are_interleaved_and_long_enough():  # tests/test_fused.py:33-40
    cos, sin = oracle.cos_sin_tables(HD, 1024, 500000.0, None)
    assert cos.shape == (1024 + 513, HD) and cos.dtype == torch.float32
    assert torch.equal(cos[:, 0::2], cos[:, 1::2]) and torch.equal(sin[:, 0::2], sin[:, 1::2])
    torch.testing.assert_close(cos[0], torch.ones(HD))


def test_relative_rotation_identity():  # tests/test_fused.py:63-73
    cos, sin = oracle.cos_sin_tables(HD, 2048, 500000.0, LLAMA3)
    T = oracle.rope_transformation_matrix(HD)
    rot = lambda x, s: x * cos[s] + (x @ T) * sin[s]
    q, k = torch.randn(HD), torch.randn(HD)
    p, s0, t = 1500, 1024, 37
    q_rel = rot(q, p) * cos[s0] - (rot(q, p) @ T) * sin[s0]
    torch.testing.assert_close(rot(q, p) @ rot(k, s0 + t), q_rel @ rot(k, t), atol=1e-3, rtol=1e-5)


def test_reference_decode_reduces_to_causal_sdpa_without_rotation():  # tests/test_fused.py:76-89
    B, nkv, nh, S, r_v = 2, 2, 4, 64, 32
    q = torch.randn(1, B, nh, HD)
    k = torch.randn(B, nkv, S, HD)
    v = torch.randn(B, nkv, S, r_v)
    cur = torch.tensor([10, 63])
    out = oracle.reference_decode(q, k, torch.eye(HD).expand(nkv, HD, HD), v, cur, torch.ones(S, HD),
                                  torch.zeros(S, HD), HD ** -0.5)
    for b in range(B):
        for h in range(nh):
            kk, vv = k[b, h // 2, : cur[b] + 1], v[b, h // 2, : cur[b] + 1]
            att = torch.softmax(q[0, b, h] @ kk.T * HD ** -0.5, -1) @ vv
            torch.testing.assert_close(out[0, b, h], att, atol=1e-5, rtol=1e-4)


def test_in_kernel_v_equals_attention_over_rebuilt_v():  # tests/test_fused.py:106-115
    B, nkv, nh, S, r_k, r_v = 1, 2, 4, 16, 32, 48
    q = torch.randn(1, B, nh, HD); k = torch.randn(B, nkv, S, r_k); u_k = torch.randn(nkv, r_k, HD)
    v_lat = torch.randn(B, nkv, S, r_v); u_v = torch.randn(nkv, r_v, HD)
    cos, sin = oracle.cos_sin_tables(HD, S, 500000.0, None)
    out = oracle.reference_decode(q, k, u_k, v_lat, torch.tensor([S - 1]), cos, sin, 1.0, u_v=u_v)
    v_full = torch.einsum("bhsr,hrd->bhsd", v_lat, u_v)
    exp = oracle.reference_decode(q, k, u_k, v_full, torch.tensor([S - 1]), cos, sin, 1.0)
    torch.testing.assert_close(out, exp, atol=1e-5, rtol=1e-4)


def test_metrics_are_relative_and_rowwise():
    ref = torch.tensor([[1.0, -1.0], [0.01, 0.01]])
    out = ref.clone()
    out[1, 0] += 0.001
    mx, mn = oracle.rel_errors(out, ref)
    assert math.isclose(mx, 0.001, rel_tol=1e-4) and math.isclose(mn, 0.001 / 2.02, rel_tol=1e-4)
    rmx, rmn = oracle.rowwise_rel_errors(out, ref)
    assert math.isclose(rmx, 0.1, rel_tol=1e-4) and math.isclose(rmn, 0.05, rel_tol=1e-4)


def test_phase2_tables_compose_chunk_base_and_relative_rows():
    """The chunk-relative rule (fused.py:1-14): exact on the first chunk (base row 0 is the identity), and for
    an fp32 table equal to the table within fp32 angle rounding; a bf16 table differs by its rounding."""
    cos, sin = oracle.cos_sin_tables(128, 4096, 500000.0, None)
    cos, sin = cos[:4096], sin[:4096]
    c2, s2 = oracle.phase2_tables(cos, sin)
    assert torch.equal(c2[:128], cos[:128]) and torch.equal(s2[:128], sin[:128])
    assert (c2 - cos).abs().max() < 5e-4 and (s2 - sin).abs().max() < 5e-4
    cb, sb = cos.bfloat16().float(), sin.bfloat16().float()
    c3, _ = oracle.phase2_tables(cb, sb)
    assert 1e-4 < (c3 - cb).abs().max() < 2e-2
