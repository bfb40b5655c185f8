"""palu_b200.convert against the reference's own outputs (golden fixtures from palu_tt/convert.py) and
the reference's convert tests restated (tests/test_convert.py). CPU only."""
import json

import numpy as np
import pytest
import torch

from palu_b200 import convert, fused
from tests.conftest import load_golden

DIM, NH, NKV, HD = 64, 4, 2, 16


def _write_dump(tmp_path, d):
    from safetensors.torch import save_file
    tensors = {k[len("dump."):]: v.contiguous() for k, v in d.items() if k.startswith("dump.")}
    save_file(tensors, str(tmp_path / "palu_lowrank.safetensors"))
    (tmp_path / "config.json").write_text(json.dumps({"head_wise_ranks": json.loads(bytes(d["ranks"]).decode())}))


@pytest.mark.parametrize("name", ["convert_mlrd_ragged", "convert_glrd_gs2", "convert_full_rank"])
def test_load_and_layer_tensors_match_reference_golden(tmp_path, name):
    d = load_golden(name)
    hd, nkv, nh, dim, rank_multiple = (int(x) for x in d["dims"])
    _write_dump(tmp_path, d)
    lr = convert.load_palu_dir(tmp_path, 1, nkv, hd, rank_multiple=rank_multiple)[0]
    for k in ("k_VT", "k_U", "v_VT", "v_U"):
        assert torch.equal(getattr(lr, k), d[f"lr.{k}"]), k
    assert lr.group_size == int(d["lr.group_size"])
    hf = {k: d[f"hf.{k}"] for k in ("q", "k", "v", "o")}
    t = convert.palu_layer_tensors(hf, lr, nh, nkv, hd)
    for k in ("wk_lat_pad", "wv_lat_pad", "u_k", "u_v", "wo_fused", "w_rot"):
        torch.testing.assert_close(t[k], d[f"t.{k}"], atol=1e-5, rtol=1e-5, msg=k)


def _hf_attn():
    return {"q": torch.randn(NH * HD, DIM), "k": torch.randn(NKV * HD, DIM), "v": torch.randn(NKV * HD, DIM),
            "o": torch.randn(DIM, NH * HD)}


def test_identity_lowrank_reproduces_stock_k_and_v():  # tests/test_convert.py:18-28
    w = _hf_attn()
    t = convert.palu_layer_tensors(w, convert.identity_lowrank(w, NKV, HD), NH, NKV, HD)
    assert torch.allclose(t["wk_lat_pad"], convert.reverse_permute(w["k"], NKV, NKV * HD, DIM), atol=1e-6)
    x = torch.randn(5, DIM)
    lat_v = x @ t["wv_lat_pad"].T
    v = torch.cat([lat_v[:, h * HD:(h + 1) * HD] @ t["u_v"][h] for h in range(NKV)], dim=-1)
    assert torch.allclose(v, x @ w["v"].T, atol=1e-5)


def test_low_rank_k_block_is_padded_latent():  # tests/test_convert.py:144-160
    w = _hf_attn()
    r_k = 8
    lr = convert.LowRank(k_VT=torch.randn(NKV, r_k, DIM), k_U=torch.randn(NKV, HD, r_k),
                         v_VT=torch.randn(NKV, HD, DIM), v_U=torch.randn(NKV, HD, HD))
    t = convert.palu_layer_tensors(w, lr, NH, NKV, HD)
    x = torch.randn(5, DIM)
    lat_k = x @ t["wk_lat_pad"].T
    for h in range(NKV):
        assert torch.count_nonzero(t["wk_lat_pad"][h * HD + r_k:(h + 1) * HD]) == 0
        w_h = convert.reverse_permute(lr.k_U[h] @ lr.k_VT[h], 1, HD, DIM)
        assert torch.allclose(lat_k[:, h * HD:h * HD + r_k] @ t["u_k"][h], x @ w_h.T, atol=1e-4)


def test_wo_fused_absorbs_u_v():  # tests/test_convert.py:200-221
    w = _hf_attn()
    r_v = 8
    v_VT, v_U = torch.randn(NKV, r_v, DIM), torch.randn(NKV, HD, r_v)
    w["v"] = torch.cat([v_U[h] @ v_VT[h] for h in range(NKV)], dim=0)
    lr = convert.LowRank(k_VT=torch.randn(NKV, HD, DIM), k_U=torch.randn(NKV, HD, HD), v_VT=v_VT, v_U=v_U)
    t = convert.palu_layer_tensors(w, lr, NH, NKV, HD)
    x = torch.randn(7, DIM)
    lat_v = (x @ t["wv_lat_pad"].T).reshape(7, NKV, HD)
    attn = torch.softmax(torch.randn(NH, 3, 7), dim=-1)
    fused_in = torch.zeros(3, NH * HD)
    for h in range(NH):
        fused_in[:, h * HD:h * HD + r_v] = attn[h] @ lat_v[:, h // (NH // NKV), :r_v]
    V = (x @ w["v"].T).reshape(7, NKV, HD)
    stock_in = torch.cat([attn[h] @ V[:, h // (NH // NKV)] for h in range(NH)], dim=-1)
    assert torch.allclose(fused_in @ t["wo_fused"].T, stock_in @ w["o"].T, atol=1e-4)


def test_unit_scale_keeps_the_product_and_is_group_aware():  # tests/test_convert.py:453-483
    g = torch.Generator().manual_seed(0)
    VT = torch.randn(4, 16, 32, generator=g)
    U = torch.randn(4, 24, 16, generator=g)
    lr = convert.LowRank(k_VT=VT[:1].repeat(4, 1, 1), k_U=U, v_VT=VT[:1].repeat(4, 1, 1), v_U=U, group_size=4)
    unit = convert.unit_scale_lowrank(lr)
    assert torch.equal(unit.k_VT[0], unit.k_VT[3])
    c = torch.sqrt((U ** 2).sum(dim=(0, 1)))
    assert torch.allclose(unit.k_U[2], U[2] * c[None, :])
    for h in range(4):
        assert torch.allclose(unit.k_U[h] @ unit.k_VT[h], lr.k_U[h] @ lr.k_VT[h], atol=1e-4)


def test_runtime_and_config_defaults():  # tests/test_convert.py:332-436
    assert convert.CONVERT_VERSION == 4
    rt = convert.PaluRuntime()
    assert rt.use_fused_k is False and rt.cs_recurrence is False and rt.fused_k_chunk is None
    assert rt.rot_mode == "dst" and rt.table_mcast is True and rt.latent_quant_in_prefill is True
    cfg = convert.PaluConfig(rank_k=[32], rank_v=[64], cache_id="x")
    assert cfg.group_size == 1 and cfg.device_tables == {}


def test_fused_table_builders_match_the_oracle():
    import oracle
    rs = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
          "original_max_position_embeddings": 8192}
    for scaling in (None, rs):
        a = fused.cos_sin_tables(128, 3000, 500000.0, scaling)
        b = oracle.cos_sin_tables(128, 3000, 500000.0, scaling)
        assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    u = torch.randn(3, 32, 128)
    assert torch.equal(fused.w_rot_from_u_k(u), oracle.w_rot_from_u_k(u))
    assert torch.equal(fused.rope_transformation_matrix(128), oracle.rope_transformation_matrix(128))
    assert [fused.chunk_size(s) for s in (96, 8192, 8224)] == [32, 512, 32]
