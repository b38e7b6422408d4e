"""Weight conversion (``convert.py``) and npz checkpoints (``checkpoint.py``).

Pinned by the reference's own torch layer: ``tests/golden/layer_d32_n16_p16.npz`` holds
a ``torch_ref.Mamba3SISOTorch`` state dict (interleaved rotary layout, ``(out, in)``
weights) and its output, so converting that state dict and running the layer oracle must
reproduce the reference module's y.  The GPU test runs the converted weights through the
CUDA layer."""

import os

import numpy as np
import pytest
import torch

from oracle import siso_oracle as O
from tests.metrics import max_rel, rel_error

F64 = torch.float64
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _golden_layer():
    with np.load(os.path.join(GOLDEN, "layer_d32_n16_p16.npz")) as z:
        g = {k: torch.from_numpy(z[k]) for k in z.files}
    sd = {k[4:].replace("__", "."): v for k, v in g.items() if k.startswith("sd__")}
    return g, sd


def _cfg_and_params(dtype=F64, device="cpu"):
    from mamba3_b200 import convert as CV

    g, sd = _golden_layer()
    cfg = CV.config_from_state_dict(sd, headdim=int(g["headdim"]), rope_fraction=float(g["rope_fraction"]),
                                    chunk=64, policy_name="f32")
    return g, sd, cfg, CV.torch_to_jax(sd, cfg, dtype=dtype, device=device)


def test_converted_reference_layer_matches_its_output():
    g, sd, cfg, p = _cfg_and_params()
    assert (cfg.d_model, cfg.d_state, cfg.headdim, cfg.nheads) == (32, 16, 16, 4)
    y, _ = O.layer_forward(p._asdict(), g["u"], d_state=cfg.d_state, headdim=cfg.headdim, nheads=cfg.nheads,
                           n_angles=cfg.n_angles, chunk=16)
    # torch_ref rounds dd_A and the angles through float32 (torch_ref.py:216, 228)
    assert max_rel(y, g["y"]) < 1e-6


def test_roundtrip_is_exact():
    from mamba3_b200 import convert as CV

    g, sd, cfg, p = _cfg_and_params(dtype=torch.float32)
    back = CV.jax_to_torch(p, cfg)
    ren = {"B_norm.weight": "B_norm_weight", "C_norm.weight": "C_norm_weight"}
    for k, v in back.items():
        assert torch.equal(v, sd[ren.get(k, k)].float()), k
    again = CV.torch_to_jax(back, cfg)
    for a, b in zip(again, p):
        assert torch.equal(a, b)


def test_mimo_and_bad_headdim_refused():
    from mamba3_b200 import convert as CV

    g, sd = _golden_layer()
    with pytest.raises(ValueError, match="headdim"):
        CV.config_from_state_dict(sd, headdim=24)
    cfg = CV.config_from_state_dict(sd, headdim=16, chunk=64)
    bad = dict(sd)
    bad["B_bias"] = torch.cat([sd["B_bias"], sd["B_bias"]], 1)
    with pytest.raises(ValueError, match="single-input"):
        CV.torch_to_jax(bad, cfg)
    del bad["B_norm_weight"]
    with pytest.raises(KeyError):
        CV.torch_to_jax(bad, cfg)


def _hf_json(**kw):
    d = {"d_model": 32, "n_layer": 2, "vocab_size": 250, "pad_vocab_size_multiple": 8, "tie_embeddings": True,
         "d_intermediate": 48, "ssm_cfg": {"layer": "Mamba3", "d_state": 16, "headdim": 16, "A_floor": 2e-4}}
    d.update(kw)
    return d


def test_config_from_hf():
    from mamba3_b200 import convert as CV

    cfg = CV.config_from_hf(_hf_json())
    assert cfg.vocab_size == 256 and cfg.n_layers == 2 and cfg.d_intermediate == 48 and cfg.tie_head
    assert cfg.siso.a_floor == 2e-4 and cfg.siso.chunk == 128 and cfg.siso.nheads == 4
    with pytest.raises(ValueError, match="MIMO"):
        CV.config_from_hf(_hf_json(ssm_cfg={"layer": "Mamba3", "mimo": True}))
    with pytest.raises(ValueError, match="attention"):
        CV.config_from_hf(_hf_json(attn_layer_idx=[1]))
    with pytest.raises(ValueError, match="Mamba3"):
        CV.config_from_hf(_hf_json(ssm_cfg={"layer": "Mamba2"}))


def _hf_state_dict(cfg, seed=0):
    """A ``MambaLMHeadModel``-shaped state dict (upstream key names and shapes)."""
    g = torch.Generator().manual_seed(seed)
    c, r = cfg.siso, lambda *s: torch.randn(*s, generator=g)
    sd = {"backbone.embedding.weight": r(cfg.vocab_size, c.d_model), "backbone.norm_f.weight": r(c.d_model)}
    for i in range(cfg.n_layers):
        m = f"backbone.layers.{i}."
        sd.update({m + "norm.weight": r(c.d_model), m + "mixer.in_proj.weight": r(c.d_in_proj, c.d_model),
                   m + "mixer.out_proj.weight": r(c.d_model, c.d_inner), m + "mixer.dt_bias": r(c.nheads),
                   m + "mixer.B_bias": r(c.nheads, 1, c.d_state), m + "mixer.C_bias": r(c.nheads, 1, c.d_state),
                   m + "mixer.B_norm.weight": r(c.d_state), m + "mixer.C_norm.weight": r(c.d_state),
                   m + "mixer.D": r(c.nheads)})
        if cfg.d_intermediate:
            sd.update({m + "norm2.weight": r(c.d_model), m + "mlp.fc1.weight": r(2 * cfg.d_intermediate, c.d_model),
                       m + "mlp.fc2.weight": r(c.d_model, cfg.d_intermediate)})
    sd["lm_head.weight"] = sd["backbone.embedding.weight"]
    return sd


def test_load_lm_state_dict():
    from mamba3_b200 import convert as CV
    from mamba3_b200 import layout as L

    cfg = CV.config_from_hf(_hf_json())
    sd = _hf_state_dict(cfg)
    p = CV.load_lm_state_dict(sd, cfg)
    c, perm = cfg.siso, L.deinterleave_perm(cfg.siso.d_state)
    assert p.head is None and torch.equal(p.embed, sd["backbone.embedding.weight"])
    b1 = p.blocks[1]
    w = sd["backbone.layers.1.mixer.in_proj.weight"].t()
    b0 = 2 * c.d_inner
    assert torch.equal(b1.siso.in_proj[:, :b0], w[:, :b0])
    assert torch.equal(b1.siso.in_proj[:, b0:b0 + c.d_state], w[:, b0:b0 + c.d_state][:, perm])
    assert torch.equal(b1.siso.in_proj[:, b0 + 2 * c.d_state:], w[:, b0 + 2 * c.d_state:])
    assert torch.equal(b1.siso.b_bias, sd["backbone.layers.1.mixer.B_bias"][:, 0][:, perm])
    assert torch.equal(b1.mlp.fc1, sd["backbone.layers.1.mlp.fc1.weight"].t())
    assert torch.equal(b1.mlp_norm_gain, sd["backbone.layers.1.norm2.weight"])
    del sd["backbone.layers.1.mlp.fc2.weight"]
    with pytest.raises(KeyError, match="fc2"):
        CV.load_lm_state_dict(sd, cfg)
    with pytest.raises(ValueError, match="embedding"):
        CV.load_lm_state_dict(_hf_state_dict(CV.config_from_hf(_hf_json(pad_vocab_size_multiple=1))), cfg)


@pytest.mark.parametrize("dtype", [None, torch.bfloat16])
@pytest.mark.parametrize("tie", [True, False])
def test_checkpoint_roundtrip(tmp_path, dtype, tie):
    from mamba3_b200 import checkpoint as CP
    from mamba3_b200 import convert as CV

    cfg = CV.config_from_hf(_hf_json(tie_embeddings=tie))
    sd = _hf_state_dict(cfg, seed=3)
    p = CV.load_lm_state_dict(sd, cfg)
    if not tie:
        p = p._replace(head=torch.randn(cfg.d_model, cfg.vocab_size))
    path = CP.save(str(tmp_path / "m"), p, cfg, dtype=dtype)
    assert path.endswith(".npz")
    with np.load(path) as z:  # readable without this package; bf16 is opaque 2-byte
        assert z["blocks.0.siso.in_proj"].dtype == (np.dtype("V2") if dtype is torch.bfloat16 else np.float32)
    q, cfg2 = CP.load(path)
    assert cfg2 == cfg
    fa, fb = CP.flat_params(p), CP.flat_params(q)
    assert [n for n, _ in fa] == [n for n, _ in fb]
    for (n, a), (_, b) in zip(fa, fb):
        want = a if dtype is None else a.to(dtype)
        assert b.dtype == want.dtype and torch.equal(b, want), n
    q32, _ = CP.load(path, dtype=torch.float32)
    assert q32.embed.dtype == torch.float32


def test_checkpoint_rejects_bad_files(tmp_path):
    from mamba3_b200 import checkpoint as CP
    from mamba3_b200 import convert as CV

    cfg = CV.config_from_hf(_hf_json(d_intermediate=0))
    p = CV.load_lm_state_dict(_hf_state_dict(cfg), cfg)
    path = CP.save(str(tmp_path / "ok.npz"), p, cfg)
    with np.load(path) as z:
        arrays = {k: z[k] for k in z.files}
    np.savez(tmp_path / "missing.npz", **{k: v for k, v in arrays.items() if k != "final_norm"})
    with pytest.raises(ValueError, match="'final_norm' not found"):
        CP.load(str(tmp_path / "missing.npz"))
    np.savez(tmp_path / "extra.npz", stray=np.zeros(3), **arrays)
    with pytest.raises(ValueError, match="does not account for"):
        CP.load(str(tmp_path / "extra.npz"))
    bad = dict(arrays)
    bad["embed"] = bad["embed"][:, :5]
    np.savez(tmp_path / "shape.npz", **bad)
    with pytest.raises(ValueError, match="shape"):
        CP.load(str(tmp_path / "shape.npz"))
    np.savez(tmp_path / "nocfg.npz", **{k: v for k, v in arrays.items() if k != CP.CONFIG_KEY})
    with pytest.raises(ValueError, match="__config__"):
        CP.load(str(tmp_path / "nocfg.npz"))
    d = CP.config_to_dict(cfg)
    d["format_version"] = CP.FORMAT_VERSION + 1
    with pytest.raises(ValueError, match="newer"):
        CP.config_from_dict(d)


@pytest.mark.gpu
def test_converted_reference_layer_on_gpu():
    from mamba3_b200 import layer as LY

    g, sd, cfg, p = _cfg_and_params(dtype=torch.float32, device="cuda")
    y, _ = LY.mamba3_siso_layer(p, g["u"].float().cuda(), cfg)
    assert rel_error(y, g["y"]) < 1e-5
