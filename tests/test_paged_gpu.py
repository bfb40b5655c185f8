"""Paged latent caches on the GPU: palu_decode_attn_paged and palu_append_latents_paged.

The caches are [n_blocks, n_groups, block_size, r] and a page table [B, blocks per row] maps each row's
logical blocks to physical ones (the stock paged flash-decode convention the reference's plan names,
HANDOFF.md:126-127). Bars (written here):

* bit-identical to palu_decode_attn on contiguous caches holding the same latents at the same logical
  positions: the kernels, the tile order and the split are the same, only the addresses differ;
* against the oracle (reference_decode over the gathered positions): the decode bar, max-abs relative
  <= 2e-2 and mean-abs relative <= 1e-3, globally and per (row, head) on the fp32 output;
* the paged append: bit-identical to the oracle's paged_append.

Page tables are random permutations of the physical blocks (consecutive logical blocks scattered), with
spare blocks no row maps. Rows end anywhere in a block (cur_pos 0, 63, 64, 127, 128, S/2, S-1, random).
"""
import pytest
import torch

import oracle
from tests.test_decode_gpu import _bf, _inputs, assert_close

pytestmark = pytest.mark.gpu

SCALE = 128 ** -0.5


@pytest.fixture(params=["tc", "mma"])
def kernel(request, cuda):
    from palu_b200 import _lib
    _lib.set_kernel(_lib.PALU_KERNEL_TC if request.param == "tc" else _lib.PALU_KERNEL_MMA)
    yield request.param
    _lib.set_kernel(_lib.PALU_KERNEL_AUTO)


def _decode(dev, q, k, v, u_k, cos, sin, pos, S, u_v=None, page_table=None, splits=0):
    """One decode call through the library (fp32 output): contiguous caches, or paged with page_table."""
    from palu_b200 import fused
    w_rot = fused.w_rot_from_u_k(u_k.float()).to(dev, torch.bfloat16)
    cs = fused.pack_cs_table(fused.cs_table(cos, sin, S).to(dev, torch.bfloat16))
    out = fused.decode(q[0].to(dev, torch.bfloat16), k.to(dev, torch.bfloat16), v.to(dev, torch.bfloat16), w_rot, cs,
                       pos.to(dev, torch.int32), u_k_ld=256, u_v=None if u_v is None else u_v.to(dev, torch.bfloat16),
                       out_dtype=torch.float32, splits=splits,
                       page_table=None if page_table is None else page_table.to(dev))
    torch.cuda.synchronize()
    assert fused.workspace_status() == 0, "a bounded device wait expired"
    return out.cpu()


def _oracle(q, k_lat, u_k, v_lat, pos, cos, sin, u_v, n_groups):
    gs = 8 // n_groups
    return oracle.reference_decode(q, oracle.expand_groups(k_lat, gs), u_k, oracle.expand_groups(v_lat, gs), pos,
                                   cos, sin, SCALE, u_v=u_v)[0]


def _paged(g, k_lat, v_lat, bs, spare=5):
    B, _, S, _ = k_lat.shape
    per_row = (S + bs - 1) // bs
    n_blocks = B * per_row + spare
    pt = oracle.shuffled_page_table(B, per_row, n_blocks, g)
    return pt, oracle.paged_scatter(k_lat, pt, n_blocks, bs), oracle.paged_scatter(v_lat, pt, n_blocks, bs)


SHAPES = [(64, 64, 8, False), (128, 96, 8, False), (64, 64, 2, True)]  # (r_k, r_v, latent groups, u_v)


@pytest.mark.parametrize("bs", [16, 32, 64, 128])
@pytest.mark.parametrize("r_k,r_v,n_groups,uv", SHAPES, ids=["mlrd64", "mlrd128x96", "glrd_gs4"])
def test_paged_equals_contiguous_and_oracle(cuda, kernel, bs, r_k, r_v, n_groups, uv):
    g = torch.Generator().manual_seed(bs * 7 + r_k + r_v + n_groups)
    B, S = 7, 1024
    q, k_lat, u_k, v_lat, u_v, pos, cos, sin = _inputs(g, B, 8, 32, S, r_k, r_v, n_groups=n_groups, uv=uv)
    pt, kp, vp = _paged(g, k_lat, v_lat, bs)
    want = _decode(cuda, q, k_lat, v_lat, u_k, cos, sin, pos, S, u_v=u_v)
    got = _decode(cuda, q, kp, vp, u_k, cos, sin, pos, S, u_v=u_v, page_table=pt)
    assert torch.equal(got, want), f"paged differs from contiguous: max {(got - want).abs().max():.3e}"
    assert_close(got, _oracle(q, k_lat, u_k, v_lat, pos, cos, sin, u_v, n_groups), f"bs={bs}")


def test_wide_latents_paged_on_the_mma_kernel(cuda):
    """Rank-256 grouped latents (outside the tcgen05 envelope) through the mma.sync kernel's paged loads."""
    g = torch.Generator().manual_seed(256)
    B, S, bs = 3, 768, 32
    q, k_lat, u_k, v_lat, u_v, pos, cos, sin = _inputs(g, B, 8, 32, S, 256, 256, n_groups=2, uv=True)
    pt, kp, vp = _paged(g, k_lat, v_lat, bs)
    want = _decode(cuda, q, k_lat, v_lat, u_k, cos, sin, pos, S, u_v=u_v)
    got = _decode(cuda, q, kp, vp, u_k, cos, sin, pos, S, u_v=u_v, page_table=pt)
    assert torch.equal(got, want)
    assert_close(got, _oracle(q, k_lat, u_k, v_lat, pos, cos, sin, u_v, 2), "r=256 paged")


def test_entries_past_each_row_are_never_read(cuda, kernel):
    """Table entries beyond a row's last position are garbage (-1, huge, out of range): the output is the
    one the clean table gives, so the kernels read no entry past ceil((cur_pos + 1) / block_size)."""
    g = torch.Generator().manual_seed(41)
    B, S, bs = 6, 1024, 16
    q, k_lat, u_k, v_lat, _, pos, cos, sin = _inputs(g, B, 8, 32, S, 64, 64)
    pt, kp, vp = _paged(g, k_lat, v_lat, bs)
    want = _decode(cuda, q, kp, vp, u_k, cos, sin, pos, S, page_table=pt)
    dirty = pt.clone()
    junk = torch.tensor([-1, 1 << 30, -(1 << 30), pt.numel() + 100], dtype=torch.int32)
    for b in range(B):
        used = (int(pos[b]) + bs) // bs  # blocks covering positions 0..cur_pos
        n = dirty.shape[1] - used
        dirty[b, used:] = junk[torch.arange(n) % 4]
    got = _decode(cuda, q, kp, vp, u_k, cos, sin, pos, S, page_table=dirty)
    assert torch.equal(got, want)


def test_unmapped_block_reads_zero_latents(cuda, kernel):
    """An entry outside [0, n_blocks) inside a row's range reads as zero latents (no access outside the
    caches): the output matches the oracle over the gathered, zero-filled positions."""
    g = torch.Generator().manual_seed(43)
    B, S, bs = 4, 512, 32
    q, k_lat, u_k, v_lat, _, pos, cos, sin = _inputs(g, B, 8, 32, S, 64, 64)
    pos[:] = torch.tensor([S - 1, 300, 100, 33], dtype=torch.int32)
    pt, kp, vp = _paged(g, k_lat, v_lat, bs)
    n_blocks = kp.shape[0]
    pt[0, 3], pt[1, 0], pt[2, 1], pt[3, 1] = n_blocks, -7, n_blocks + 1000, -1
    got = _decode(cuda, q, kp, vp, u_k, cos, sin, pos, S, page_table=pt)
    ref = _oracle(q, oracle.paged_gather(kp, pt, S), u_k, oracle.paged_gather(vp, pt, S), pos, cos, sin, None, 8)
    assert_close(got, ref, "unmapped blocks")


def test_paged_append_matches_oracle(cuda):
    """Decode-step appends through the page table, including rows at cur_pos -1 and max_seq (skipped) and
    a row whose entry is outside the caches (dropped), equal the oracle's paged_append bit for bit."""
    from palu_b200 import fused
    g = torch.Generator().manual_seed(44)
    B, G, r_k, r_v, bs, per_row = 5, 2, 48, 96, 32, 6
    S = per_row * bs
    n_blocks = B * per_row + 3
    pt = oracle.shuffled_page_table(B, per_row, n_blocks, g)
    pt[4, 2] = n_blocks + 9
    kc = _bf(torch.randn(n_blocks, G, bs, r_k, generator=g))
    vc = _bf(torch.randn(n_blocks, G, bs, r_v, generator=g))
    kd, vd = kc.to(cuda, torch.bfloat16), vc.to(cuda, torch.bfloat16)
    for step, pos in enumerate(([0, 31, 32, S - 1, 70], [-1, S, 100, 5, 64 + 3], [1, 2, 3, 4, 95])):
        pos = torch.tensor(pos, dtype=torch.int32)
        nk = _bf(torch.randn(B, G, r_k, generator=g))
        nv = _bf(torch.randn(B, G, r_v, generator=g))
        fused.append_latents(nk.to(cuda), nv.to(cuda), pos.to(cuda), kd, vd, page_table=pt.to(cuda))
        oracle.paged_append(kc, nk, pos, pt, S)
        oracle.paged_append(vc, nv, pos, pt, S)
        torch.cuda.synchronize()
        assert torch.equal(kd.float().cpu(), kc) and torch.equal(vd.float().cpu(), vc), f"step {step}"


def test_paged_layer_equals_contiguous_layer(cuda):
    """PaluAttention with paged caches (tt_transformers' paged_attention_config / page_table arguments):
    a prefill through the page table and three decode steps give the contiguous layer's outputs."""
    from palu_b200.attention import PaluAttention, PagedAttentionConfig
    from palu_b200.convert import LowRank
    g = torch.Generator().manual_seed(45)
    dim, nh, nkv, r_k, r_v, B, P, S, bs = 512, 8, 4, 64, 32, 3, 40, 256, 32
    wq = torch.randn(nh * 128, dim, generator=g) * dim ** -0.5
    wo = torch.randn(dim, nh * 128, generator=g) * (nh * 128) ** -0.5
    lr = LowRank(k_VT=torch.randn(nkv, r_k, dim, generator=g) * dim ** -0.5,
                 k_U=torch.randn(nkv, 128, r_k, generator=g) * r_k ** -0.5,
                 v_VT=torch.randn(nkv, r_v, dim, generator=g) * dim ** -0.5,
                 v_U=torch.randn(nkv, 128, r_v, generator=g) * r_v ** -0.5)
    kw = dict(max_batch=B, max_seq=S, device="cuda")
    flat = PaluAttention(wq, wo, lr, nh, nkv, **kw)
    per_row = S // bs
    cfg = PagedAttentionConfig(block_size=bs, max_num_blocks=B * per_row + 4)
    paged = PaluAttention(wq, wo, lr, nh, nkv, paged_attention_config=cfg, **kw)
    pt = oracle.shuffled_page_table(B, per_row, cfg.max_num_blocks, g).to(cuda)
    x = torch.randn(B, P, dim, generator=g).to(cuda)
    assert torch.equal(paged.forward_prefill(x, page_table=pt), flat.forward_prefill(x))
    for step in range(3):
        xd = torch.randn(B, dim, generator=g).to(cuda)
        pos = torch.tensor([P + step, P - 1 + 2 * step, 7 * step], dtype=torch.int32, device=cuda)
        assert torch.equal(paged.forward_decode(xd, pos, page_table=pt), flat.forward_decode(xd, pos)), step


def test_paged_decoder_step_and_graph_replay(cuda):
    """The decoder over paged caches: a prefill and an eager greedy step give the contiguous decoder's
    logits, and one step captured as a CUDA graph (page table in a captured buffer) replays the eager
    step's tokens."""
    from palu_b200.attention import PagedAttentionConfig
    from palu_b200.model import DecoderConfig, PaluDecoder
    cfg = DecoderConfig(dim=512, n_layers=2, n_heads=4, n_kv_heads=2, ffn_dim=768, vocab=300)
    B, P, S, bs = 2, 16, 64, 16
    pc = PagedAttentionConfig(block_size=bs, max_num_blocks=B * S // bs + 3)
    kw = dict(max_batch=B, max_seq=S, seed=5, device="cuda", proj_dtype=torch.float32)
    flat = PaluDecoder(cfg, [(32, 64), (48, 32)], **kw)
    paged = PaluDecoder(cfg, [(32, 64), (48, 32)], paged_attention_config=pc, **kw)
    pt = oracle.shuffled_page_table(B, S // bs, pc.max_num_blocks, torch.Generator().manual_seed(8)).to(cuda)
    tokens = torch.randint(0, cfg.vocab, (B, P), generator=torch.Generator().manual_seed(9))
    want = flat.prefill_logits(tokens)
    assert torch.equal(paged.prefill_logits(tokens, page_table=pt), want)
    nxt = want.argmax(-1)
    pos = torch.full((B,), P, dtype=torch.int32, device=cuda)
    assert torch.equal(paged.decode_logits(nxt, pos, page_table=pt), flat.decode_logits(nxt, pos))
    graph = paged.capture_decode(B, page_table=pt)
    pos1 = pos + 1
    eager = paged.decode_step(nxt, pos1, page_table=pt)
    graph.tokens.copy_(nxt)
    graph.pos.copy_(pos1)
    replayed = graph.replay().clone()
    torch.cuda.synchronize()
    assert torch.equal(eager, replayed)
