"""Paged latent caches without a GPU: the oracle's page-table model, the layer's host logic with CPU
models of the two device ops, and the C ABI's page-table validation (which fails before any CUDA call)."""
import ctypes

import pytest
import torch

import oracle
from tests.test_attention_layer import _cpu_ops


def test_scatter_gather_round_trip_and_unmapped_zeros():
    g = torch.Generator().manual_seed(1)
    B, G, S, r, bs = 3, 2, 100, 16, 32  # S not a whole number of blocks
    x = torch.randn(B, G, S, r, generator=g)
    per_row = -(-S // bs)
    pt = oracle.shuffled_page_table(B, per_row, B * per_row + 2, g)
    paged = oracle.paged_scatter(x, pt, B * per_row + 2, bs)
    assert torch.equal(oracle.paged_gather(paged, pt, S), x)
    pt[1, 2] = -1
    got = oracle.paged_gather(paged, pt, S)
    assert torch.equal(got[1, :, 64:96], torch.zeros(G, 32, r)) and torch.equal(got[0], x[0])


def test_paged_append_equals_contiguous_append():
    g = torch.Generator().manual_seed(2)
    B, G, S, r, bs = 4, 2, 64, 8, 16
    contig = torch.randn(B, G, S, r, generator=g)
    pt = oracle.shuffled_page_table(B, S // bs, B * S // bs, g)
    paged = oracle.paged_scatter(contig, pt, B * S // bs, bs)
    new = torch.randn(B, G, r, generator=g)
    pos = torch.tensor([0, 17, -1, S], dtype=torch.int32)
    oracle.paged_append(paged, new, pos, pt, S)
    contig[0, :, 0], contig[1, :, 17] = new[0], new[1]
    assert torch.equal(oracle.paged_gather(paged, pt, S), contig)


def _cpu_paged_ops(layer):
    """The CPU models of _cpu_ops, reading and writing through the page table."""
    _cpu_ops(layer)
    append_c, attend_c = layer.append_op, layer.attend_op

    def append(new_k, new_v, pos, kc, vc, page_table):
        S = page_table.shape[1] * kc.shape[2]
        oracle.paged_append(kc, new_k.to(kc.dtype), pos, page_table, S)
        oracle.paged_append(vc, new_v.to(vc.dtype), pos, page_table, S)

    def attend(q, kc, w_rot, cs_tab, vc, head_dim_v, pos, page_table_tensor, **kw):
        S = page_table_tensor.shape[1] * kc.shape[2]
        return attend_c(q, oracle.paged_gather(kc, page_table_tensor, S), w_rot, cs_tab,
                        oracle.paged_gather(vc, page_table_tensor, S), head_dim_v, pos, **kw)
    layer.append_op, layer.attend_op = append, attend


@pytest.mark.parametrize("gs", [1, 2])
def test_paged_layer_equals_contiguous_layer_on_cpu_models(gs):
    """Prefill through the page table (per batch and per user) and decode steps: the paged layer's outputs
    equal the contiguous layer's, so the host side moves every latent to the position the op reads."""
    from palu_b200.attention import PaluAttention, PagedAttentionConfig
    from palu_b200.convert import LowRank
    g = torch.Generator().manual_seed(3 + gs)
    dim, nh, nkv, r_k, r_v, B, P, S, bs = 256, 4, 2, 32, 16, 3, 20, 64, 16
    rep = lambda t: t.repeat_interleave(gs, 0)[:nkv]  # G-LRD: a group's factors repeated per head
    lr = LowRank(k_VT=rep(torch.randn(nkv // gs, r_k, dim, generator=g) * dim ** -0.5),
                 k_U=torch.randn(nkv, 128, r_k, generator=g) * r_k ** -0.5,
                 v_VT=rep(torch.randn(nkv // gs, r_v, dim, generator=g) * dim ** -0.5),
                 v_U=torch.randn(nkv, 128, r_v, generator=g) * r_v ** -0.5)
    wq = torch.randn(nh * 128, dim, generator=g) * dim ** -0.5
    wo = torch.randn(dim, nh * 128, generator=g) * (nh * 128) ** -0.5
    kw = dict(max_batch=B, max_seq=S, device="cpu")
    flat = PaluAttention(wq, wo, lr, nh, nkv, **kw)
    cfg = PagedAttentionConfig(block_size=bs, max_num_blocks=B * S // bs + 3)
    paged = PaluAttention(wq, wo, lr, nh, nkv, paged_attention_config=cfg, **kw)
    _cpu_ops(flat)
    _cpu_paged_ops(paged)
    pt = oracle.shuffled_page_table(B, S // bs, cfg.max_num_blocks, g)
    x = torch.randn(B, P, dim, generator=g)
    assert torch.equal(paged.forward_prefill(x, page_table=pt), flat.forward_prefill(x))
    xu = torch.randn(1, 1, P - 3, dim, generator=g)  # one user's prompt into cache row 2
    assert torch.equal(paged.forward_prefill(xu, user_id=2, page_table=pt), flat.forward_prefill(xu, user_id=2))
    for step in range(3):
        xd = torch.randn(B, dim, generator=g)
        pos = torch.tensor([P + step, P - 3 + step, 5 * step], dtype=torch.int32)
        assert torch.equal(paged.forward_decode(xd, pos, page_table=pt), flat.forward_decode(xd, pos)), step
    with pytest.raises(RuntimeError, match="page_table"):
        paged.forward_decode(xd, pos)
    with pytest.raises(RuntimeError, match="page_table"):
        flat.forward_decode(xd, pos, page_table=pt)


def _paged_call(lib, d, pg):
    from palu_b200 import _lib
    z = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    st = lib.palu_decode_attn_paged(z, z, z, z, 256, None, z, z, ctypes.byref(pg) if pg else None, z, 0, z, 1 << 30,
                                    ctypes.byref(d), 1.0, None)
    return st, lib.palu_last_error().decode()


@pytest.mark.parametrize("change,needle", [
    (dict(block_size=24), "block_size"),
    (dict(block_size=256), "block_size"),
    (dict(table_ld=3), "table_ld"),      # 256 positions of 32 need 8 entries per row
    (dict(n_blocks=0), "n_blocks"),
    (dict(table=None), "page table"),
    (dict(table=18), "aligned"),
    ("none", "pages is NULL"),
])
def test_paged_envelope_errors_from_the_abi(change, needle):
    from palu_b200 import _lib
    lib = _lib.load()
    d = _lib.dims(2, 32, 8, 8, 64, 64, 256)
    base = dict(table=16, table_ld=8, block_size=32, n_blocks=64)
    if change != "none":
        base.update(change)
    pg = None if change == "none" else _lib.PageTable(**base)
    st, msg = _paged_call(lib, d, pg)
    assert st == _lib.PALU_ERR_INVALID and needle in msg, msg
    if pg is not None:
        z = ctypes.c_void_p(16)
        st = lib.palu_append_latents_paged(z, z, z, ctypes.byref(pg), z, z, ctypes.byref(d), None)
        assert st == _lib.PALU_ERR_INVALID and needle in lib.palu_last_error().decode()


def test_paged_call_applies_the_decode_envelope():
    """A valid page table does not bypass the op's own checks (here an unsupported r_k)."""
    from palu_b200 import _lib
    lib = _lib.load()
    d = _lib.dims(2, 32, 8, 8, 40, 64, 256)
    st, msg = _paged_call(lib, d, _lib.PageTable(16, 8, 32, 64))
    assert st == _lib.PALU_ERR_INVALID and "r_k" in msg, msg


def test_paged_decoder_equals_contiguous_decoder_on_cpu_models():
    """The decoder with paged caches in every layer (one page table for the batch) gives the contiguous
    decoder's logits for a prefill and two greedy decode steps."""
    from palu_b200.attention import PagedAttentionConfig
    from palu_b200.model import DecoderConfig, PaluDecoder
    cfg = DecoderConfig(dim=256, n_layers=2, n_heads=4, n_kv_heads=2, ffn_dim=384, vocab=200)
    B, P, S, bs = 2, 12, 48, 16
    pc = PagedAttentionConfig(block_size=bs, max_num_blocks=B * S // bs + 2)
    kw = dict(max_batch=B, max_seq=S, seed=5, device="cpu", proj_dtype=torch.float32)
    flat = PaluDecoder(cfg, [(32, 16), (16, 32)], **kw)
    paged = PaluDecoder(cfg, [(32, 16), (16, 32)], paged_attention_config=pc, **kw)
    for L in flat.layers:
        _cpu_ops(L["attn"])
    for L in paged.layers:
        _cpu_paged_ops(L["attn"])
    pt = oracle.shuffled_page_table(B, S // bs, pc.max_num_blocks, torch.Generator().manual_seed(6))
    tokens = torch.randint(0, cfg.vocab, (B, P), generator=torch.Generator().manual_seed(7))
    want = flat.prefill_logits(tokens)
    assert torch.equal(paged.prefill_logits(tokens, page_table=pt), want)
    nxt = want.argmax(-1)
    for step in range(2):
        pos = torch.full((B,), P + step, dtype=torch.int32)
        want = flat.decode_logits(nxt, pos)
        assert torch.equal(paged.decode_logits(nxt, pos, page_table=pt), want), step
        nxt = want.argmax(-1)
