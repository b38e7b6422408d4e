"""Weight conversion between upstream PyTorch Mamba-3 SISO checkpoints and this package's
`layer.SISOParams` / `model.LMParams` (``mamba3_pallas/convert.py``).

An upstream mixer differs from `layer.SISOParams` in three ways, all undone here:

* ``nn.Linear`` weights are ``(out, in)``; the layer applies ``u @ W`` with ``(in, out)``.
* Upstream rotates adjacent state channels (2j, 2j+1); the kernels rotate the half-split
  pairs (j, N/2 + j).  `layout.deinterleave_perm` maps one onto the other.  It is applied
  to every tensor on the state axis: the B and C column blocks of in_proj, the two bias
  tables and the two norm gains (``convert.py:112-160``).  dt_bias, D and out_proj carry
  no state axis and pass through; q~.k~ is unchanged because rotations are orthogonal.
* Upstream biases are ``(H, R, N)`` with the MIMO rank R; SISO needs R == 1.

`torch_to_jax` / `jax_to_torch` keep the reference's names for one mixer (the "jax" side is
this package's parameter tuple); `load_lm_state_dict` maps a whole ``MambaLMHeadModel``
state dict (``convert.py:176-330``).
"""

from __future__ import annotations

from typing import Any, Dict, Mapping

import torch

from . import layer as LY
from . import layout as L

MIXER_PREFIX = "backbone.layers.{i}.mixer."


def _f32(x: Any) -> torch.Tensor:
    """Any array-like (bf16 tensors included) as a float32 CPU tensor."""
    if isinstance(x, torch.Tensor):
        return x.detach().to("cpu", torch.float32)
    return torch.as_tensor(x).to(torch.float32)


def config_from_state_dict(sd: Mapping[str, Any], headdim: int = 64, **overrides) -> LY.SISOConfig:
    """``convert.py:60-95``: a `layer.SISOConfig` from one mixer's shapes.  headdim is not
    visible in the weights (only nheads * headdim), so it is an argument."""
    d_in_proj, d_model = _f32(sd["in_proj.weight"]).shape
    b_bias = _f32(sd["B_bias"])
    nheads, d_state = b_bias.shape[0], b_bias.shape[-1]
    d_inner = nheads * headdim
    if d_inner % d_model != 0:
        raise ValueError(f"inner width {nheads} heads x {headdim} = {d_inner} does not divide evenly by "
                         f"d_model {d_model}: pass the checkpoint's real headdim")
    cfg = LY.SISOConfig(d_model=d_model, d_state=d_state, headdim=headdim, expand=d_inner // d_model, **overrides)
    if cfg.d_in_proj != d_in_proj:
        raise ValueError(f"in_proj has {d_in_proj} output rows; a single-input (SISO) mixer with headdim "
                         f"{headdim} would have {cfg.d_in_proj}. Multi-input (MIMO) checkpoints are not supported.")
    return cfg


def _norm_gain(sd: Mapping[str, Any], prefix: str) -> torch.Tensor:
    for key in (f"{prefix}_norm.weight", f"{prefix}_norm_weight"):
        if key in sd:
            return _f32(sd[key])
    raise KeyError(f"missing {prefix} norm weight ({prefix}_norm.weight)")


def _bias(sd: Mapping[str, Any], prefix: str) -> torch.Tensor:
    arr = _f32(sd[f"{prefix}_bias"])
    if arr.dim() == 3:
        if arr.shape[1] != 1:
            raise ValueError(f"{prefix}_bias carries {arr.shape[1]} input ranks; only single-input (rank 1) "
                             f"mixers are supported")
        arr = arr[:, 0]
    return arr


def torch_to_jax(sd: Mapping[str, Any], cfg: LY.SISOConfig, dtype=torch.float32, device="cpu") -> LY.SISOParams:
    """``convert.py:98-161``: one mixer's state dict -> `layer.SISOParams` in the kernels'
    half-split layout.  Accepts norm gains as ``B_norm.weight`` (upstream) or
    ``B_norm_weight`` (the reference's torch module)."""
    n = cfg.d_state
    perm = L.deinterleave_perm(n)
    in_proj = _f32(sd["in_proj.weight"]).t().contiguous()
    out_proj = _f32(sd["out_proj.weight"]).t().contiguous()
    b0 = 2 * cfg.d_inner  # column order [z, x, B, C, dt, A, trap, angles]
    for start in (b0, b0 + n):
        in_proj[:, start:start + n] = in_proj[:, start:start + n][:, perm]
    to = dict(dtype=dtype, device=device)
    return LY.SISOParams(
        in_proj=in_proj.to(**to), out_proj=out_proj.to(**to), dt_bias=_f32(sd["dt_bias"]).to(**to),
        b_norm_weight=_norm_gain(sd, "B")[perm].to(**to), c_norm_weight=_norm_gain(sd, "C")[perm].to(**to),
        b_bias=_bias(sd, "B")[:, perm].to(**to), c_bias=_bias(sd, "C")[:, perm].to(**to),
        d_skip=_f32(sd["D"]).to(**to))


def jax_to_torch(params: LY.SISOParams, cfg: LY.SISOConfig) -> Dict[str, torch.Tensor]:
    """``convert.py:164-189``: the inverse of `torch_to_jax`, float32 CPU tensors in
    upstream's shapes (biases ``(H, 1, N)``) and channel order."""
    n = cfg.d_state
    inv = L.interleave_perm(n)
    in_proj = _f32(params.in_proj).clone()
    b0 = 2 * cfg.d_inner
    for start in (b0, b0 + n):
        in_proj[:, start:start + n] = in_proj[:, start:start + n][:, inv]
    return {
        "in_proj.weight": in_proj.t().contiguous(),
        "out_proj.weight": _f32(params.out_proj).t().contiguous(),
        "dt_bias": _f32(params.dt_bias),
        "B_norm.weight": _f32(params.b_norm_weight)[inv],
        "C_norm.weight": _f32(params.c_norm_weight)[inv],
        "B_bias": _f32(params.b_bias)[:, inv][:, None, :].contiguous(),
        "C_bias": _f32(params.c_bias)[:, inv][:, None, :].contiguous(),
        "D": _f32(params.d_skip),
    }


# Aliases with this package's vocabulary.
torch_to_params = torch_to_jax
params_to_torch = jax_to_torch


def config_from_hf(cfg_json: Mapping[str, Any], **overrides):
    """``convert.py:214-276``: a released ``config.json`` -> `model.LMConfig`.  The vocab
    is padded up to ``pad_vocab_size_multiple`` (the embedding's real width); the chunk
    is a tiling choice, not a weight shape, and defaults to 128."""
    from . import model as M

    ssm = dict(cfg_json.get("ssm_cfg", {}))
    layer_name = ssm.pop("layer", "Mamba3")
    if layer_name != "Mamba3":
        raise ValueError(f"ssm_cfg.layer is {layer_name!r}, expected 'Mamba3'")
    if ssm.get("mimo", False) or ssm.get("mimo_rank", 1) not in (1, None):
        raise ValueError("this checkpoint is MIMO; only SISO is implemented")
    if cfg_json.get("attn_layer_idx"):
        raise ValueError(f"checkpoint has attention layers at {cfg_json['attn_layer_idx']}; "
                         "hybrid attention/SSM stacks are not implemented")
    if ssm.get("ngroups", 1) != 1:
        raise ValueError(f"ngroups={ssm['ngroups']}, only ngroups=1 (SISO) is implemented")
    vocab = int(cfg_json["vocab_size"])
    mult = int(cfg_json.get("pad_vocab_size_multiple", 1) or 1)
    if vocab % mult:
        vocab += mult - vocab % mult
    kw: Dict[str, Any] = {
        "d_model": int(cfg_json["d_model"]),
        "d_state": int(ssm.get("d_state", 128)),
        "headdim": int(ssm.get("headdim", 64)),
        "expand": int(ssm.get("expand", 2)),
        "rope_fraction": float(ssm.get("rope_fraction", 0.5)),
        "chunk": 128,
    }
    for src, dst in (("A_floor", "a_floor"), ("dt_min", "dt_min"), ("dt_max", "dt_max"),
                     ("dt_init_floor", "dt_init_floor")):
        if src in ssm:
            kw[dst] = float(ssm[src])
    kw.update({k: v for k, v in overrides.items() if k != "d_intermediate"})
    return M.LMConfig(vocab_size=vocab, n_layers=int(cfg_json["n_layer"]), siso=LY.SISOConfig(**kw),
                      tie_head=bool(cfg_json.get("tie_embeddings", True)),
                      d_intermediate=int(cfg_json.get("d_intermediate", 0)))


def load_lm_state_dict(sd: Mapping[str, Any], cfg, dtype=torch.float32, device="cpu"):
    """``convert.py:279-330``: a ``MambaLMHeadModel`` state dict -> `model.LMParams`.
    Strict: a key the config implies but the checkpoint lacks raises KeyError."""
    from . import model as M

    to = dict(dtype=dtype, device=device)

    def get(key: str) -> torch.Tensor:
        if key not in sd:
            raise KeyError(f"checkpoint is missing {key!r}")
        return _f32(sd[key])

    embed = get("backbone.embedding.weight")
    if tuple(embed.shape) != (cfg.vocab_size, cfg.d_model):
        raise ValueError(f"embedding is {tuple(embed.shape)}, config implies {(cfg.vocab_size, cfg.d_model)}; "
                         "check pad_vocab_size_multiple")
    blocks = []
    for i in range(cfg.n_layers):
        pre = MIXER_PREFIX.format(i=i)
        mixer = {k[len(pre):]: sd[k] for k in sd if k.startswith(pre)}
        if not mixer:
            raise KeyError(f"no keys under {pre!r}; is this a Mamba-3 checkpoint?")
        siso = torch_to_jax(mixer, cfg.siso, dtype, device)
        mlp = mlp_norm = None
        if cfg.d_intermediate:
            mlp = M.MLPParams(fc1=get(f"backbone.layers.{i}.mlp.fc1.weight").t().contiguous().to(**to),
                              fc2=get(f"backbone.layers.{i}.mlp.fc2.weight").t().contiguous().to(**to))
            mlp_norm = get(f"backbone.layers.{i}.norm2.weight").to(**to)
        blocks.append(M.BlockParams(norm_gain=get(f"backbone.layers.{i}.norm.weight").to(**to), siso=siso,
                                    mlp_norm_gain=mlp_norm, mlp=mlp))
    # a tied head shares storage with the embedding upstream: read lm_head only when untied
    head = None if cfg.tie_head else get("lm_head.weight").t().contiguous().to(**to)
    return M.LMParams(embed=embed.to(**to), blocks=blocks, final_norm=get("backbone.norm_f.weight").to(**to),
                      head=head)


def load_pretrained(repo_id: str, dtype=torch.float32, revision=None, device="cpu", **cfg_overrides):
    """``convert.py:333-356``: fetch ``config.json`` and ``pytorch_model.bin`` from the
    Hugging Face Hub and convert them.  Needs ``huggingface_hub`` and network access."""
    import json

    try:
        from huggingface_hub import hf_hub_download
    except ImportError as e:  # not part of this image
        raise ImportError("load_pretrained needs huggingface_hub; convert a local state dict with "
                          "load_lm_state_dict instead") from e
    with open(hf_hub_download(repo_id, "config.json", revision=revision)) as fh:
        cfg = config_from_hf(json.load(fh), **cfg_overrides)
    sd = torch.load(hf_hub_download(repo_id, "pytorch_model.bin", revision=revision), map_location="cpu",
                    weights_only=True)
    return load_lm_state_dict(sd, cfg, dtype, device), cfg
