"""Self-describing ``.npz`` checkpoints of `model.LMParams` (``mamba3_pallas/checkpoint.py``).

One array per parameter under a dotted name (``embed``, ``blocks.0.norm_gain``,
``blocks.0.siso.in_proj``, ``blocks.0.mlp.fc1``, ``final_norm``, ``head``), plus a
``__config__`` entry holding the `model.LMConfig` and each array's dtype name as JSON
bytes.  No pickle.  bfloat16, which numpy lacks, is stored as opaque 2-byte values (numpy
``|V2``) and restored from the recorded name, as the reference's writer does, so files
written by either side load in the other.
"""

from __future__ import annotations

import dataclasses
import json
from typing import Any, Dict, List, Tuple

import numpy as np
import torch

from . import layer as LY
from . import model as M

#: Bumped if the on-disk layout changes in a way old readers cannot handle.
FORMAT_VERSION = 1
#: The entry holding the JSON config (not a valid parameter name).
CONFIG_KEY = "__config__"

_DT_NAMES = {torch.float32: "float32", torch.bfloat16: "bfloat16", torch.float16: "float16", torch.float64: "float64"}


def flat_params(params: M.LMParams) -> List[Tuple[str, torch.Tensor]]:
    """``checkpoint.py:46-69``: the parameter tree as (dotted name, tensor) pairs in tree
    order; absent optional entries (no MLP, tied head) contribute nothing."""
    out: List[Tuple[str, torch.Tensor]] = [("embed", params.embed)]
    for i, b in enumerate(params.blocks):
        out.append((f"blocks.{i}.norm_gain", b.norm_gain))
        out.extend((f"blocks.{i}.siso.{f}", getattr(b.siso, f)) for f in LY.SISOParams._fields)
        if b.mlp_norm_gain is not None:
            out.append((f"blocks.{i}.mlp_norm_gain", b.mlp_norm_gain))
        if b.mlp is not None:
            out.extend((f"blocks.{i}.mlp.{f}", getattr(b.mlp, f)) for f in M.MLPParams._fields)
    out.append(("final_norm", params.final_norm))
    if params.head is not None:
        out.append(("head", params.head))
    return out


def config_to_dict(cfg: M.LMConfig) -> Dict[str, Any]:
    """``checkpoint.py:72-95``."""
    c = cfg.siso
    return {
        "format_version": FORMAT_VERSION,
        "vocab_size": cfg.vocab_size,
        "n_layers": cfg.n_layers,
        "tie_head": cfg.tie_head,
        "d_intermediate": cfg.d_intermediate,
        "siso": {f.name: getattr(c, f.name) for f in dataclasses.fields(LY.SISOConfig)},
    }


def config_from_dict(d: Dict[str, Any]) -> M.LMConfig:
    """``checkpoint.py:98-120``: unknown ``siso`` keys are dropped (a newer writer), missing
    ones take `layer.SISOConfig`'s defaults; a newer format version raises."""
    got = d.get("format_version", 0)
    if got > FORMAT_VERSION:
        raise ValueError(f"checkpoint format version {got} is newer than this package supports ({FORMAT_VERSION})")
    fields = {f.name for f in dataclasses.fields(LY.SISOConfig)}
    return M.LMConfig(vocab_size=int(d["vocab_size"]), n_layers=int(d["n_layers"]),
                      siso=LY.SISOConfig(**{k: v for k, v in d["siso"].items() if k in fields}),
                      tie_head=bool(d["tie_head"]), d_intermediate=int(d.get("d_intermediate", 0)))


def _shape_template(cfg: M.LMConfig) -> M.LMParams:
    """The parameter tree of `model.init_lm` as shape-only (meta) tensors."""
    c, e = cfg.siso, lambda *s: torch.empty(*s, device="meta")
    di = cfg.d_intermediate
    blocks = [M.BlockParams(
        norm_gain=e(c.d_model),
        siso=LY.SISOParams(in_proj=e(c.d_model, c.d_in_proj), out_proj=e(c.d_inner, c.d_model), dt_bias=e(c.nheads),
                           b_norm_weight=e(c.d_state), c_norm_weight=e(c.d_state), b_bias=e(c.nheads, c.d_state),
                           c_bias=e(c.nheads, c.d_state), d_skip=e(c.nheads)),
        mlp_norm_gain=e(c.d_model) if di else None,
        mlp=M.MLPParams(fc1=e(c.d_model, 2 * di), fc2=e(di, c.d_model)) if di else None) for _ in range(cfg.n_layers)]
    return M.LMParams(embed=e(cfg.vocab_size, c.d_model), blocks=blocks, final_norm=e(c.d_model),
                      head=None if cfg.tie_head else e(c.d_model, cfg.vocab_size))


def _to_numpy(t: torch.Tensor) -> np.ndarray:
    t = t.detach().to("cpu").contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view("V2")
    return t.numpy()


def save(path: str, params: M.LMParams, cfg: M.LMConfig, dtype: torch.dtype = None) -> str:
    """``checkpoint.py:134-172``: write ``params`` and ``cfg``; returns the path written
    (numpy appends ``.npz`` when it is missing).  ``dtype`` casts every array first."""
    arrays: Dict[str, np.ndarray] = {}
    dtypes: Dict[str, str] = {}
    for name, t in flat_params(params):
        if dtype is not None:
            t = t.to(dtype)
        if t.dtype not in _DT_NAMES:
            raise ValueError(f"{name}: unsupported dtype {t.dtype}")
        arrays[name] = _to_numpy(t)
        dtypes[name] = _DT_NAMES[t.dtype]
    meta = {**config_to_dict(cfg), "dtypes": dtypes}
    arrays[CONFIG_KEY] = np.frombuffer(json.dumps(meta).encode("utf-8"), dtype=np.uint8)
    np.savez(path, **arrays)
    return path if path.endswith(".npz") else path + ".npz"


def load(path: str, dtype: torch.dtype = None, device="cpu") -> Tuple[M.LMParams, M.LMConfig]:
    """``checkpoint.py:175-206``: read a checkpoint; the stored config rebuilds the tree, a
    missing, extra or mis-shaped array raises ValueError."""
    with np.load(path, allow_pickle=False) as z:
        if CONFIG_KEY not in z.files:
            raise ValueError(f"{path} has no {CONFIG_KEY} entry; not a mamba3-siso checkpoint")
        meta = json.loads(bytes(z[CONFIG_KEY]).decode("utf-8"))
        cfg = config_from_dict(meta)
        stored = meta.get("dtypes", {})
        template = _shape_template(cfg)
        names = [n for n, _ in flat_params(template)]
        got: Dict[str, torch.Tensor] = {}
        for (name, ref) in flat_params(template):
            if name not in z.files:
                raise ValueError(f"parameter {name!r} not found in {path}")
            a = z[name]
            if tuple(a.shape) != tuple(ref.shape):
                raise ValueError(f"{name}: checkpoint has shape {a.shape}, config implies {tuple(ref.shape)}")
            if a.dtype.kind == "V":
                if stored.get(name) != "bfloat16" or a.dtype.itemsize != 2:
                    raise ValueError(f"{name}: opaque dtype {a.dtype} without a bfloat16 record")
                t = torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
            else:
                t = torch.from_numpy(np.ascontiguousarray(a))
            got[name] = t.to(device=device, dtype=dtype if dtype is not None else t.dtype)
        extra = set(z.files) - {CONFIG_KEY} - set(names)
        if extra:
            raise ValueError(f"{path} holds arrays the config does not account for: {sorted(extra)}")
    blocks = []
    for i, b in enumerate(template.blocks):
        siso = LY.SISOParams(*(got[f"blocks.{i}.siso.{f}"] for f in LY.SISOParams._fields))
        mlp = None if b.mlp is None else M.MLPParams(*(got[f"blocks.{i}.mlp.{f}"] for f in M.MLPParams._fields))
        blocks.append(M.BlockParams(norm_gain=got[f"blocks.{i}.norm_gain"], siso=siso,
                                    mlp_norm_gain=got.get(f"blocks.{i}.mlp_norm_gain"), mlp=mlp))
    return M.LMParams(embed=got["embed"], blocks=blocks, final_norm=got["final_norm"], head=got.get("head")), cfg
