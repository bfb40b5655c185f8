"""The Palu decoder (palu_b200/model.py) against a reference decoder built from the oracle's layer.

The reference: per layer the oracle's ``PaluRefAttention`` (reference.py:14-55; HF rotate-half RoPE, fp32)
between RMSNorms, a fp32 SwiGLU MLP and residuals, then RMSNorm and the LM head, all from the decoder's own
checkpoint-layout weights (``keep_source``), with the oracle's ``device_rounding``: the latent caches in
bf16, and in a decode step q rounded to bf16 after RoPE and K rotated with the bf16 table, which are the
values the device path stores (without them the roundings alone move the logits by a few 1e-3). A tiny
config (2 layers, 4 query / 2 KV heads, dim 512; one model with one rank pair per layer, one with ranks
per KV head zero-padded per layer as the reference's loader pads them): a 16-token prefill, then two
greedy-fed decode steps.

Tolerance (written here): the north star's, max-abs relative <= 2e-2 and mean-abs relative <= 1e-3 on the
fp32 logits.

The CPU test runs the decoder with its two device ops per layer replaced by CPU models (the oracle's
reference_decode and a cache write), which checks the model algebra without a GPU; the GPU tests run the
CUDA library, and replay one decode step as a CUDA graph.
"""
import pytest
import torch

import oracle
from oracle.metrics import rel_errors
from tests.test_attention_layer import _cpu_ops

MAX_REL, MEAN_REL = 2e-2, 1e-3
B, P = 2, 16
# per layer: one (r_k, r_v) for every KV head, or per-head ranks (K ranks, V ranks) padded per layer
RANKS = {"per_layer": [(32, 64), (48, 32)], "per_head": [([32, 48], [64, 16]), ([96, 16], [32, 128])]}


def _model(device, ranks="per_layer"):
    from palu_b200.model import DecoderConfig, PaluDecoder
    cfg = DecoderConfig(dim=512, n_layers=2, n_heads=4, n_kv_heads=2, ffn_dim=768, vocab=300)
    m = PaluDecoder(cfg, RANKS[ranks], max_batch=B, max_seq=40, seed=5, device=device,
                    proj_dtype=torch.float32, keep_source=True)
    return cfg, m


class _RefDecoder:
    """fp32 reference decoder from the model's source weights (test infrastructure)."""

    def __init__(self, cfg, m):
        hf = dict(hidden_size=cfg.dim, num_attention_heads=cfg.n_heads, num_key_value_heads=cfg.n_kv_heads,
                  num_hidden_layers=cfg.n_layers, intermediate_size=cfg.ffn_dim, vocab_size=cfg.vocab,
                  max_position_embeddings=131072, rope_theta=cfg.rope_theta, rope_scaling=cfg.rope_scaling)
        self.cfg = cfg
        self.layers = []
        for L in m.layers:
            s = L["src"]
            lr = s["lowrank"]
            cpu_lr = type(lr)(k_VT=lr.k_VT.cpu(), k_U=lr.k_U.cpu(), v_VT=lr.v_VT.cpu(), v_U=lr.v_U.cpu())
            attn = oracle.PaluRefAttention(hf, {"q": s["wq"].cpu(), "o": s["wo"].cpu()}, cpu_lr, device_rounding=True)
            self.layers.append((attn, s["w1"].cpu().float(), s["w3"].cpu().float(), s["w2"].cpu().float()))
        self.embed, self.lm_head = m.embed.cpu().float(), m.lm_head.cpu().float()

    def forward(self, tokens, start_pos):
        """tokens [B, S] at positions start_pos.. -> logits [B, S, vocab]."""
        norm = lambda x: x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.cfg.norm_eps)
        h = self.embed[tokens]
        for attn, w1, w3, w2 in self.layers:
            h = h + attn.forward(norm(h), start_pos)
            x = norm(h)
            h = h + (torch.nn.functional.silu(x @ w1.T) * (x @ w3.T)) @ w2.T
        return norm(h) @ self.lm_head.T


def _check(got, want, what):
    mx, mn = rel_errors(got.float().cpu(), want.float())
    assert mx <= MAX_REL and mn <= MEAN_REL, f"{what}: max {mx:.3e} mean {mn:.3e}"


def _run(m, ref):
    g = torch.Generator().manual_seed(9)
    tokens = torch.randint(0, m.cfg.vocab, (B, P), generator=g)
    _check(m.prefill_logits(tokens), ref.forward(tokens, 0)[:, -1], "prefill")
    nxt = ref.forward(tokens, 0)[:, -1].argmax(-1)  # fresh reference caches are rebuilt at start_pos 0
    for step in range(2):
        pos = torch.full((B,), P + step, dtype=torch.int32)
        want = ref.forward(nxt[:, None], P + step)[:, 0]
        _check(m.decode_logits(nxt, pos), want, f"decode step {step}")
        nxt = want.argmax(-1)
    return nxt


@pytest.mark.parametrize("ranks", list(RANKS))
def test_decoder_matches_reference_decoder_on_cpu_models(ranks):
    cfg, m = _model("cpu", ranks)
    for L in m.layers:
        _cpu_ops(L["attn"])
    _run(m, _RefDecoder(cfg, m))


def test_mixed_ranks_are_seeded_and_legal():
    from palu_b200.model import mixed_head_ranks, mixed_ranks, padded_rank
    r = mixed_ranks(32, seed=3)
    assert r == mixed_ranks(32, seed=3) and len(r) == 32
    assert all(rk in (32, 48, 64, 96, 128) and rv in (32, 48, 64, 96, 128) for rk, rv in r)
    assert len(set(r)) > 1
    h = mixed_head_ranks(32, 8, seed=7)
    assert h == mixed_head_ranks(32, 8, seed=7) and len(h) == 32
    assert all(len(k) == 8 and len(v) == 8 and set(k + v) <= {32, 48, 64, 96, 128} for k, v in h)
    assert padded_rank([32, 48]) == 64 and padded_rank([96, 32]) == 96 and padded_rank([128]) == 128
    # per head AND per layer: most layers hold a 128 somewhere (P = 1 - 0.8^8 per side)
    assert sum(padded_rank(k) == 128 for k, _ in h) > 16


def test_per_head_ranks_pad_with_zero_factors():
    """A per-head rank below the layer width leaves that head's extra VT rows and U columns zero."""
    cfg, m = _model("cpu", "per_head")
    lr = m.layers[0]["src"]["lowrank"]
    assert lr.k_VT.shape[1] == 64 and lr.v_VT.shape[1] == 64
    assert lr.k_VT[0, 32:].abs().sum() == 0 and lr.k_U[0, :, 32:].abs().sum() == 0
    assert lr.v_VT[1, 16:].abs().sum() == 0 and lr.v_U[1, :, 16:].abs().sum() == 0
    assert lr.k_VT[1, :48].abs().sum() > 0 and lr.k_VT[1, 48:].abs().sum() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("ranks", list(RANKS))
def test_decoder_matches_reference_decoder_on_gpu(cuda, ranks):
    cfg, m = _model("cuda", ranks)
    _run(m, _RefDecoder(cfg, m))


@pytest.mark.gpu
def test_decode_graph_replays_the_eager_step(cuda):
    """One decode step captured as a CUDA graph gives the eager step's next tokens (rewriting the same
    latents at the same positions)."""
    cfg, m = _model("cuda")
    tokens = torch.randint(0, cfg.vocab, (B, P), generator=torch.Generator().manual_seed(4))
    m.prefill_logits(tokens)
    graph = m.capture_decode(B)  # its warm-up runs at position -1 and writes no cache row
    tok = torch.tensor([7, 123], device=cuda)
    pos = torch.full((B,), P, dtype=torch.int32, device=cuda)
    eager = m.decode_step(tok, pos)
    graph.tokens.copy_(tok)
    graph.pos.copy_(pos)
    replayed = graph.replay().clone()
    torch.cuda.synchronize()
    assert torch.equal(eager, replayed)


def _tp_rank(rank, world, port, out_q):
    import datetime
    import os
    import sys
    from pathlib import Path
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "tt-cadlab_b200")]
    import torch.distributed as dist
    from palu_b200.model import DecoderConfig, PaluDecoder
    from tests.test_attention_layer import _cpu_ops as cpu_ops
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        cfg = DecoderConfig(dim=512, n_layers=2, n_heads=4, n_kv_heads=2, ffn_dim=768, vocab=300)
        m = PaluDecoder(cfg, [(32, 64), (48, 32)], max_batch=B, max_seq=40, seed=5, device="cpu",
                        proj_dtype=torch.float32, rank=rank, world=world)
        for L in m.layers:
            cpu_ops(L["attn"])
        tokens = torch.randint(0, cfg.vocab, (B, P), generator=torch.Generator().manual_seed(9))
        pre = m.prefill_logits(tokens)
        dec = m.decode_logits(pre.argmax(-1), torch.full((B,), P, dtype=torch.int32))
        if rank == 0:  # numpy arrays travel by value (a shared-memory tensor can race this process's exit)
            out_q.put((pre.numpy(), dec.numpy()))
    finally:
        dist.destroy_process_group()


def test_two_rank_tensor_parallel_decoder_equals_one_rank():
    """KV heads and the MLP hidden dimension split over 2 gloo ranks: the all-reduced logits equal the
    unsharded model's (same weights, same CPU ops)."""
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    pre2, dec2 = (torch.from_numpy(a) for a in q.get(timeout=180))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    cfg, m = _model("cpu")
    for L in m.layers:
        _cpu_ops(L["attn"])
    tokens = torch.randint(0, cfg.vocab, (B, P), generator=torch.Generator().manual_seed(9))
    pre1 = m.prefill_logits(tokens)
    dec1 = m.decode_logits(pre1.argmax(-1), torch.full((B,), P, dtype=torch.int32))
    # Each rank's projections are GEMMs of other shapes (other summation orders), and the latents are then
    # rounded to bf16 in the caches, which flips an occasional last bit: agreement to ~1e-5, bar 1e-4.
    for got, want in ((pre2, pre1), (dec2, dec1)):
        mx, mn = rel_errors(got, want)
        assert mx < 1e-4 and mn < 1e-4, (mx, mn)


@pytest.mark.gpu
def test_fused_norm_and_swiglu_kernels_match_tensor_ops(cuda):
    """palu_add_rms_norm and palu_swiglu against the tensor ops they replace: the residual sum bit for bit,
    the bf16 outputs within one bf16 rounding step (the fused kernels sum the squares in another order)."""
    from palu_b200 import fused
    g = torch.Generator().manual_seed(3)
    N, D, f = 64, 4096, 1792
    h = torch.randn(N, D, generator=g).to(cuda)
    delta = torch.randn(N, D, generator=g).to(cuda)
    w = (1 + 0.1 * torch.randn(D, generator=g)).to(cuda)
    want_h = h + delta
    want = torch.nn.functional.rms_norm(want_h, (D,), w, 1e-5).to(torch.bfloat16)
    got = fused.add_rms_norm(h, delta, w, 1e-5)
    assert torch.equal(h, want_h)
    rel = ((got.float() - want.float()).abs() / want.float().abs().clamp_min(1e-3)).max().item()
    assert rel <= 2 ** -7, rel
    d16 = delta.to(torch.bfloat16)  # a bf16 delta (a GEMM's output) is widened exactly while it is added
    want_h = h + d16.float()
    fused.add_rms_norm(h, d16, w, 1e-5)
    assert torch.equal(h, want_h)
    gu = torch.randn(N, 2 * f, generator=g).to(cuda, torch.bfloat16)
    want = torch.nn.functional.silu(gu[:, :f]) * gu[:, f:]
    got = fused.swiglu(gu, f)
    rel = ((got.float() - want.float()).abs() / want.float().abs().clamp_min(1e-3)).max().item()
    assert rel <= 2 ** -7, rel


@pytest.mark.gpu
def test_bf16_decoder_fused_elementwise_matches_tensor_ops(cuda):
    """A bf16 decoder step through the fused norm / SwiGLU kernels against the same step in tensor ops:
    logits within the layer bar (the two paths round the normalized activations separately)."""
    cfg = DecoderConfig_small()
    from palu_b200.model import PaluDecoder
    m = PaluDecoder(cfg, [(32, 64), (48, 32)], max_batch=B, max_seq=40, seed=5, device="cuda")
    tokens = torch.randint(0, cfg.vocab, (B, P), generator=torch.Generator().manual_seed(9))
    nxt = m.prefill_logits(tokens).argmax(-1)
    pos = torch.full((B,), P, dtype=torch.int32, device=cuda)
    fast = m.decode_logits(nxt, pos)
    m._fused_elementwise = lambda: False
    slow = m.decode_logits(nxt, pos)
    _check(fast, slow.cpu(), "fused vs tensor-op decoder step")


def DecoderConfig_small():
    from palu_b200.model import DecoderConfig
    return DecoderConfig(dim=512, n_layers=2, n_heads=4, n_kv_heads=2, ffn_dim=768, vocab=300)
