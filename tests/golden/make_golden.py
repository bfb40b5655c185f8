"""Generate the golden fixtures in this directory by running the REFERENCE's own Python code.

Run where the reference tree is mounted (it is not present on GPU boxes; the fixtures travel instead):

    PYTHONPATH=.:tests/golden python tests/golden/make_golden.py /path/to/tt-cadlab

It imports ``palu_tt.fused``, ``palu_tt.convert`` and ``palu_tt.reference`` from that tree, with the three
tt-metal helpers the reference does not vendor supplied by ``_ref_stubs`` (this repository's restatements),
and saves inputs + reference outputs as ``.npz``. It also runs the reference's own CPU tests
(tests/test_fused.py, tests/test_reference.py, tests/test_convert.py) against those stand-ins and records
the outcome in ``PINNING.md``.

Inputs follow the reference's device-test recipe (tests/test_palu_sdpa_device.py:45-55, 218-231):
bf16-rounded q ~ N(0,1), latents ~ N(0,1), U ~ N(0, 1/r); positions include S-1, 0, 127 and 128 so
that the first row, both sides of a 128-token tile boundary and the full cache are covered.
"""
import json
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
THETA = 500000.0
LLAMA3 = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
          "original_max_position_embeddings": 8192}


def _bf(t):
    return t.to(torch.bfloat16).float()


def _np(d):
    return {k: (v.numpy() if isinstance(v, torch.Tensor) else np.asarray(v)) for k, v in d.items()}


def _positions(g, B, S):
    pos = torch.randint(0, S, (B,), generator=g)
    pos[0] = S - 1
    if B >= 4:
        pos[1], pos[2], pos[3] = 0, 127, 128
    return pos.to(torch.int32)


def decode_case(fused, seed, B, nkv, nh, S, r_k, r_v, group_size=1, identity=False, rope_scaling=LLAMA3):
    g = torch.Generator().manual_seed(seed)
    n_lat = nkv // group_size
    q = _bf(torch.randn(1, B, nh, 128, generator=g))
    k_lat = _bf(torch.randn(B, n_lat, S, r_k, generator=g))
    v_lat = _bf(torch.randn(B, n_lat, S, r_v, generator=g))
    if identity:
        u_k = torch.eye(128).expand(nkv, 128, 128).contiguous()
    else:
        u_k = _bf(torch.randn(nkv, r_k, 128, generator=g) / r_k ** 0.5)
    u_v = _bf(torch.randn(nkv, r_v, 128, generator=g) / r_v ** 0.5) if group_size > 1 else None
    pos = _positions(g, B, S)
    cos, sin = fused.cos_sin_tables(128, S, THETA, rope_scaling)
    cos, sin = _bf(cos), _bf(sin)
    scale = 128 ** -0.5
    k_h = k_lat.repeat_interleave(group_size, dim=1)
    v_h = v_lat.repeat_interleave(group_size, dim=1)
    out = fused.reference_decode(q, k_h, u_k, v_h, pos, cos, sin, scale, u_v=u_v)
    d = dict(q=q, k_lat=k_lat, v_lat=v_lat, u_k=u_k, cur_pos=pos, cos=cos[:S], sin=sin[:S],
             scale=np.float32(scale), group_size=np.int32(group_size), out=out)
    if u_v is not None:
        d["u_v"] = u_v
    return d


def long_case(fused, seed, B, nkv, nh, S, r_k, r_v, positions):
    """A long-context decode (the sweep's mixed-path layer at 32k positions) through the reference's own
    reference_decode. The inputs are NOT stored: they are regenerated from ``seed`` by
    ``oracle.seeded_decode_inputs`` (tens of MB of latents), and their checksums are stored so that the
    consumer can verify it regenerated the same tensors before comparing against ``out``."""
    import oracle
    q, k_lat, v_lat, u_k, _ = oracle.seeded_decode_inputs(seed, B, nkv, nh, S, r_k, r_v)
    pos = torch.tensor(positions, dtype=torch.int32)
    cos, sin = fused.cos_sin_tables(128, S, THETA, LLAMA3)
    cos, sin = _bf(cos), _bf(sin)
    out = fused.reference_decode(q, k_lat, u_k, v_lat, pos, cos, sin, 128 ** -0.5)
    return dict(seed=np.int64(seed), dims=np.array([B, nkv, nh, S, r_k, r_v], dtype=np.int64), cur_pos=pos,
                checksums=oracle.input_checksums(q, k_lat, v_lat, u_k), scale=np.float32(128 ** -0.5), out=out)


def layer_case(reference, convert, seed):
    """PaluRefAttention (reference.py:14-55) on a small llama3-scaled layer: prefill 24 tokens, then
    two decode steps. head_dim 128 so the same fixture drives the CUDA decode path."""
    g = torch.Generator().manual_seed(seed)
    nh, nkv, hd, r_k, r_v = 4, 2, 128, 32, 64
    dim = nh * hd
    cfg = dict(hidden_size=dim, num_attention_heads=nh, num_key_value_heads=nkv, num_hidden_layers=1,
               intermediate_size=128, vocab_size=256, max_position_embeddings=131072, rope_theta=THETA,
               rope_scaling=dict(LLAMA3), rms_norm_eps=1e-5, tie_word_embeddings=False)
    w = {"q": _bf(torch.randn(dim, dim, generator=g) / dim ** 0.5),
         "o": _bf(torch.randn(dim, dim, generator=g) / dim ** 0.5)}
    lr = convert.LowRank(k_VT=_bf(torch.randn(nkv, r_k, dim, generator=g) / dim ** 0.5),
                         k_U=_bf(torch.randn(nkv, hd, r_k, generator=g) / r_k ** 0.5),
                         v_VT=_bf(torch.randn(nkv, r_v, dim, generator=g) / dim ** 0.5),
                         v_U=_bf(torch.randn(nkv, hd, r_v, generator=g) / r_v ** 0.5))
    ref = reference.PaluRefAttention(cfg, w, lr)
    B, P = 2, 24
    x_pre = _bf(torch.randn(B, P, dim, generator=g))
    x_d1 = _bf(torch.randn(B, 1, dim, generator=g))
    x_d2 = _bf(torch.randn(B, 1, dim, generator=g))
    y_pre = ref.forward(x_pre, 0)
    y_d1 = ref.forward(x_d1, P)
    y_d2 = ref.forward(x_d2, P + 1)
    return dict(cfg=np.frombuffer(json.dumps(cfg).encode(), dtype=np.uint8), wq=w["q"], wo=w["o"],
                k_VT=lr.k_VT, k_U=lr.k_U, v_VT=lr.v_VT, v_U=lr.v_U, x_pre=x_pre, x_d1=x_d1, x_d2=x_d2,
                y_pre=y_pre, y_d1=y_d1, y_d2=y_d2)


def convert_case(convert, seed, group_size, ranks_k, ranks_v, hd=32, nkv=4, nh=8, dim=64, rank_multiple=32):
    """A Palu dump (Palu's on-disk layout, test_convert.py:349-363) -> load_palu_dir -> palu_layer_tensors."""
    from safetensors.torch import save_file
    g = torch.Generator().manual_seed(seed)
    n_groups = nkv // group_size
    tensors, ranks = {}, {}
    for proj, rl in (("k_proj", ranks_k), ("v_proj", ranks_v)):
        assert len(rl) == n_groups
        key = f"model.layers.0.self_attn.{proj}"
        tensors[f"{key}.VT.weight"] = torch.randn(sum(rl), dim, generator=g)
        for gi, r in enumerate(rl):
            tensors[f"{key}.U.{gi}.weight"] = torch.randn(group_size * hd, r, generator=g)
        ranks[key] = list(rl)
    hf = {"q": torch.randn(nh * hd, dim, generator=g), "k": torch.randn(nkv * hd, dim, generator=g),
          "v": torch.randn(nkv * hd, dim, generator=g), "o": torch.randn(dim, nh * hd, generator=g)}
    with tempfile.TemporaryDirectory() as td:
        save_file(tensors, str(Path(td) / "palu_lowrank.safetensors"))
        (Path(td) / "config.json").write_text(json.dumps({"head_wise_ranks": ranks}))
        lr = convert.load_palu_dir(Path(td), 1, nkv, hd, rank_multiple=rank_multiple)[0]
    t = convert.palu_layer_tensors(hf, lr, nh, nkv, hd)
    d = {f"dump.{k}": v for k, v in tensors.items()}
    d.update({f"hf.{k}": v for k, v in hf.items()})
    d.update({"lr.k_VT": lr.k_VT, "lr.k_U": lr.k_U, "lr.v_VT": lr.v_VT, "lr.v_U": lr.v_U,
              "lr.group_size": np.int32(lr.group_size)})
    d.update({f"t.{k}": v for k, v in t.items()})
    d["ranks"] = np.frombuffer(json.dumps(ranks).encode(), dtype=np.uint8)
    d["dims"] = np.array([hd, nkv, nh, dim, rank_multiple], dtype=np.int32)
    return d


def main(ref_root: str):
    ref_root = str(Path(ref_root).resolve())
    sys.path[:0] = [str(REPO), str(HERE), ref_root]
    import _ref_stubs
    _ref_stubs.install()
    from palu_tt import convert, fused, reference

    cases = {
        # absorbed V (M-LRD), S not a multiple of the tile, tile-boundary positions
        "decode_mlrd_r64": decode_case(fused, 1, B=4, nkv=2, nh=8, S=320, r_k=64, r_v=64),
        # the sweep's mixed-path layer shape: r_k 32 / r_v 128, all 32/8 heads
        "decode_mlrd_rk32_rv128": decode_case(fused, 2, B=3, nkv=8, nh=32, S=200, r_k=32, r_v=128),
        # identity factorisation (U = I, rank 128): must equal plain GQA decode
        "decode_identity_r128": decode_case(fused, 3, B=2, nkv=2, nh=8, S=192, r_k=128, r_v=128, identity=True),
        # G-LRD: one group of 4 KV heads shares a 128/256-wide latent, V rebuilt per head
        "decode_glrd_gs4": decode_case(fused, 4, B=4, nkv=4, nh=16, S=256, r_k=128, r_v=256, group_size=4),
        # no rope scaling (the reference device tests' tables, rope_scaling=None)
        "decode_mlrd_plain_rope": decode_case(fused, 5, B=2, nkv=2, nh=8, S=130, r_k=96, r_v=64, rope_scaling=None),
    }
    for name, d in cases.items():
        np.savez_compressed(HERE / f"{name}.npz", **_np(d))
    # long context: 2 rows of the sweep's r_k 32 / r_v 128 layer over 32768 positions (inputs from the seed)
    np.savez_compressed(HERE / "decode_long_rk32_rv128_s32768.npz",
                        **_np(long_case(fused, 12, B=2, nkv=8, nh=32, S=32768, r_k=32, r_v=128,
                                        positions=[32767, 20000])))
    np.savez_compressed(HERE / "layer_mlrd_llama3.npz", **_np(layer_case(reference, convert, 6)))
    np.savez_compressed(HERE / "convert_mlrd_ragged.npz",
                        **_np(convert_case(convert, 7, 1, [16, 8, 32, 24], [32, 32, 16, 8], rank_multiple=8)))
    np.savez_compressed(HERE / "convert_glrd_gs2.npz",
                        **_np(convert_case(convert, 8, 2, [24, 16], [32, 8], rank_multiple=8)))
    np.savez_compressed(HERE / "convert_full_rank.npz",
                        **_np(convert_case(convert, 9, 1, [32] * 4, [32] * 4, rank_multiple=32)))

    # The reference's own CPU tests against the restated tt-metal helpers.
    env = dict(PYTHONDONTWRITEBYTECODE="1", PYTHONPATH=f"{HERE}:{REPO}:{ref_root}",
               PATH="/usr/bin:/bin:/usr/local/bin")
    import os
    env = {**os.environ, **env}
    r = subprocess.run([sys.executable, "-m", "pytest", "-p", "_ref_stubs", "-p", "no:cacheprovider", "-q",
                        "tests/test_fused.py", "tests/test_reference.py", "tests/test_convert.py"],
                       cwd=ref_root, env=env, capture_output=True, text=True)
    summary = [ln for ln in r.stdout.splitlines() if " passed" in ln or " failed" in ln or "error" in ln]
    (HERE / "PINNING.md").write_text(
        "# Oracle pinning record\n\n"
        "Written by `tests/golden/make_golden.py`.\n\n"
        "The reference's own CPU tests, run against this repository's restatements of the three\n"
        "tt-metal helpers the reference does not vendor (`get_rot_transformation_mat`,\n"
        "`compute_gather_cos_sin`, `reverse_permute`; see `_ref_stubs.py`):\n\n"
        "```\npython -m pytest -p _ref_stubs -q tests/test_fused.py tests/test_reference.py tests/test_convert.py\n"
        + "\n".join(summary[-3:]) + "\n```\n\n"
        "Fixtures (inputs and the reference's outputs, produced by the reference's own functions):\n\n"
        + "\n".join(f"* `{p.name}`" for p in sorted(HERE.glob("*.npz"))) + "\n")
    print("\n".join(summary[-3:]))
    return r.returncode


if __name__ == "__main__":
    import os
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PALU_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_golden.py <reference tree root>  (or set PALU_REFERENCE_ROOT)")
    sys.exit(main(root))
