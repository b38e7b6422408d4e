"""Forward chunked scan through libm3siso.so.

`siso_forward` keeps the signature and return convention of
``mamba3_pallas/kernel_fwd.py:204-388`` (preprocessed boundary).  `siso_forward_raw` is
the fused boundary of ``siso.py:154-216``: raw in_proj streams in, preprocessing done
inside the kernel.
"""

from __future__ import annotations

import ctypes

from typing import NamedTuple, Optional

import torch

from . import _capi as C
from . import _tensors as T
from . import layout as L


class ForwardResiduals(NamedTuple):
    """``kernel_fwd.py:41-52``: ybar ``(B,H,L,P)`` f32, chunk_states ``(B,H,nc,P,N)``."""

    ybar: torch.Tensor
    chunk_states: torch.Tensor


def _kernel_code(kernel: str) -> int:
    """``"auto"`` (tensor cores where they apply), ``"generic"``, ``"tensorcore"`` or
    ``"tensorcore_v1"`` (the two-sequence tensor-core forward, kept for comparison)."""
    codes = {"auto": C.M3_KERNEL_AUTO, "generic": C.M3_KERNEL_GENERIC, "tensorcore": C.M3_KERNEL_TENSORCORE,
             "tensorcore_v1": C.M3_KERNEL_TENSORCORE_V1}
    if kernel not in codes:
        raise ValueError(f"kernel must be one of {sorted(codes)}, got {kernel!r}")
    return codes[kernel]


def _dims(q, v, n_angles, chunk) -> C.M3Dims:
    b, l, n = q.shape
    return C.M3Dims(b, l, v.shape[1], n, v.shape[3], n_angles, chunk)


def _check_shapes(q, k, v, z):
    if q.dim() != 3 or q.shape != k.shape:
        raise ValueError(f"q {tuple(q.shape)} and k {tuple(k.shape)} must match and be (B, L, N)")
    b, l, _ = q.shape
    if v.dim() != 4 or v.shape[0] != b or v.shape[2] != l:
        raise ValueError(f"unexpected v shape {tuple(v.shape)}")
    if z is not None and z.shape != v.shape:
        raise ValueError(f"z {tuple(z.shape)} must match v {tuple(v.shape)}")


def siso_forward(q, k, v, adt, gamma, scale, phi, q_bias, k_bias, d_skip=None, z=None,
                 seed_ssm=None, seed_k=None, seed_v=None, seed_coef=None, chunk: int = 128,
                 dtype_policy: str = "bf16", save_residuals: bool = False, out_y=None, kernel: str = "auto",
                 interpret=False, device_kind=None):
    """Chunked forward at the preprocessed boundary.  ``interpret`` / ``device_kind`` are
    the reference's TPU options (Pallas interpret mode, TPU generation); they are accepted
    and have no effect here.

    Returns ``(y, final_ssm, final_k, final_v)`` and `ForwardResiduals` when
    ``save_residuals`` (``kernel_fwd.py:245-248``).  ``final_k`` is rotated but unscaled.
    """
    L.validate_chunk(chunk)
    T.require_cuda(q, k, v)
    _check_shapes(q, k, v, z)
    b, l, n = q.shape
    h, p = v.shape[1], v.shape[3]
    nr = phi.shape[-1]
    nc = L.num_chunks(l, chunk)
    for name, t in (("adt", adt), ("gamma", gamma), ("scale", scale)):
        if tuple(t.shape) != (b, h, l):
            raise ValueError(f"{name} must be (B, H, L) = {(b, h, l)}, got {tuple(t.shape)}")
    if tuple(phi.shape) != (b, h, l, nr):
        raise ValueError(f"phi must be (B, H, L, Nr) = {(b, h, l, nr)}, got {tuple(phi.shape)}")
    seeds = (seed_ssm, seed_k, seed_v, seed_coef)
    if any(s is not None for s in seeds) and not all(s is not None for s in seeds):
        raise ValueError("seed_ssm, seed_k, seed_v and seed_coef must be given together")
    dt_io = v.dtype if v.dtype in (torch.bfloat16, torch.float32) else torch.float32
    q, k, v, z = (T.inner_contig(t, dt_io) for t in (q, k, v, z))
    adt, gamma, scale, phi = (T.f32dense(t) for t in (adt, gamma, scale, phi))
    qb, kb, dsk = T.f32dense(q_bias), T.f32dense(k_bias), T.f32dense(d_skip)
    s_ssm, s_k, s_v, s_c = (T.f32dense(t) for t in seeds)
    dev = q.device
    y = out_y if out_y is not None else torch.empty(b, h, l, p, dtype=dt_io, device=dev)
    fs = torch.empty(b, h, p, n, dtype=torch.float32, device=dev)
    fk = torch.empty(b, h, n, dtype=torch.float32, device=dev)
    fv = torch.empty(b, h, p, dtype=torch.float32, device=dev)
    ybar = states = None
    if save_residuals:
        ybar = torch.empty(b, h, l, p, dtype=torch.float32, device=dev)
        sdt = L.policy(dtype_policy).saved_state
        states = torch.empty(b, h, nc, p, n, dtype=sdt, device=dev)
    a = C.M3FwdArgs()
    a.dims = _dims(q, v, nr, chunk)
    a.io_dtype = T.io_dtype(dt_io)
    a.policy = T.policy_code(dtype_policy)
    a.raw = 0
    a.q, a.k, a.v, a.z = T.ptr(q), T.ptr(k), T.ptr(v), T.ptr(z)
    a.q_st, a.k_st, a.v_st = T.st_bln(q), T.st_bln(k), T.st_bhlp(v)
    if z is not None:
        a.z_st = T.st_bhlp(z)
    a.adt, a.gamma, a.scale, a.phi = T.ptr(adt), T.ptr(gamma), T.ptr(scale), T.ptr(phi)
    a.q_bias, a.k_bias, a.d_skip = T.ptr(qb), T.ptr(kb), T.ptr(dsk)
    a.seed_ssm, a.seed_k, a.seed_v, a.seed_coef = T.ptr(s_ssm), T.ptr(s_k), T.ptr(s_v), T.ptr(s_c)
    a.y, a.y_st = T.ptr(y), T.st_bhlp(y)
    a.final_ssm, a.final_k, a.final_v = T.ptr(fs), T.ptr(fk), T.ptr(fv)
    if save_residuals:
        a.ybar, a.chunk_states = T.ptr(ybar), T.ptr(states)
        a.chunk_states_dtype = T.io_dtype(states.dtype)
    a.kernel = _kernel_code(kernel)
    C.check(C.lib().m3_siso_fwd(a, T.stream_handle(dev)))
    if save_residuals:
        return y, fs, fk, fv, ForwardResiduals(ybar=ybar, chunk_states=states)
    return y, fs, fk, fv


def siso_forward_raw(q, k, v, dt_raw, a_raw, trap_raw, angles, dt_bias, q_bias, k_bias,
                     d_skip=None, z=None, seed_ssm=None, seed_k=None, seed_v=None, seed_phi=None,
                     a_floor: float = 1e-4, chunk: int = 128, dtype_policy: str = "bf16",
                     y_out: Optional[torch.Tensor] = None, kernel: str = "auto",
                     bwd_states: Optional[torch.Tensor] = None, return_saved: bool = False,
                     states_only: bool = False, lsplit: Optional[int] = None, rates=None):
    """Fused boundary: raw ``(B, L, H)`` dt/A/trap streams and head-shared ``(B, L, Nr)``
    angles (all may be strided views of an in_proj output).  Returns
    ``(y, final_ssm, final_k, final_v, final_phi)``.  ``y_out`` may be a strided
    ``(B, H, L, P)`` view to write into (e.g. a permuted ``(B, L, H, P)`` buffer).

    ``bwd_states``: the workspace of a later `kernel_bwd.siso_backward_raw` on the same
    inputs; when this forward runs on tensor cores it stores the chunk-start states there
    and that backward can pass ``states_ready=True``.  ``return_saved`` appends whether it
    did.  ``states_only``: no y (returned as None), only the final state -- the states-only
    variant of the tensor-core kernel; see `final_state_supported`.

    ``lsplit``: cut every sequence into that many segments scanned side by side (see
    `_forward_raw_split`); ``None`` picks it from the SM count when the batch has too few
    (b, h) sequences to fill the GPU, 1 never splits.

    ``rates``: ``(workspace, ready)`` -- a uint8 tensor of ``m3_siso_fwd_workspace_size``
    bytes for the head-shared rotary rates, and whether an earlier call on the same angles
    already filled it (the length split's two passes share one)."""
    if lsplit is None and not states_only and bwd_states is None and not return_saved:
        lsplit = _auto_split(q, v, angles, chunk, dtype_policy, kernel)
        if lsplit == 1 and _chain_fits(q, v, angles, chunk, dtype_policy, kernel):
            return _forward_raw_chain2(q, k, v, dt_raw, a_raw, trap_raw, angles, dt_bias, q_bias, k_bias, d_skip, z,
                                       seed_ssm, seed_k, seed_v, seed_phi, a_floor, chunk, dtype_policy, y_out,
                                       kernel)
    if lsplit is not None and lsplit > 1 and not states_only and bwd_states is None and not return_saved:
        return _forward_raw_split(q, k, v, dt_raw, a_raw, trap_raw, angles, dt_bias, q_bias, k_bias, d_skip, z,
                                  seed_ssm, seed_k, seed_v, seed_phi, a_floor, chunk, dtype_policy, y_out, kernel,
                                  lsplit)
    L.validate_chunk(chunk)
    T.require_cuda(q, k, v)
    _check_shapes(q, k, v, z)
    b, l, n = q.shape
    h, p = v.shape[1], v.shape[3]
    nr = angles.shape[-1]
    L.num_chunks(l, chunk)
    seeds = (seed_ssm, seed_k, seed_v)
    if any(s is not None for s in seeds) and not all(s is not None for s in seeds):
        raise ValueError("seed_ssm, seed_k and seed_v must be given together")
    dt_io = v.dtype if v.dtype in (torch.bfloat16, torch.float32) else torch.float32
    q, k, v, z = (T.inner_contig(t, dt_io) for t in (q, k, v, z))
    dt_raw, a_raw, trap_raw, angles = (T.f32c(t) for t in (dt_raw, a_raw, trap_raw, angles))
    dtb, qb, kb, dsk = (T.f32dense(t) for t in (dt_bias, q_bias, k_bias, d_skip))
    s_ssm, s_k, s_v, s_phi = (T.f32dense(t) for t in (seed_ssm, seed_k, seed_v, seed_phi))
    dev = q.device
    y = None if states_only else (y_out if y_out is not None else torch.empty(b, h, l, p, dtype=dt_io, device=dev))
    fs = torch.empty(b, h, p, n, dtype=torch.float32, device=dev)
    fk = torch.empty(b, h, n, dtype=torch.float32, device=dev)
    fv = torch.empty(b, h, p, dtype=torch.float32, device=dev)
    fphi = torch.empty(b, h, nr, dtype=torch.float32, device=dev)
    a = C.M3FwdArgs()
    a.dims = _dims(q, v, nr, chunk)
    a.io_dtype = T.io_dtype(dt_io)
    a.policy = T.policy_code(dtype_policy)
    a.raw = 1
    a.a_floor = a_floor
    a.q, a.k, a.v, a.z = T.ptr(q), T.ptr(k), T.ptr(v), T.ptr(z)
    a.q_st, a.k_st, a.v_st = T.st_bln(q), T.st_bln(k), T.st_bhlp(v)
    if z is not None:
        a.z_st = T.st_bhlp(z)
    a.dt_raw, a.a_raw, a.trap_raw = T.ptr(dt_raw), T.ptr(a_raw), T.ptr(trap_raw)
    if dt_raw.stride() != a_raw.stride() or dt_raw.stride() != trap_raw.stride():
        dt_raw, a_raw, trap_raw = dt_raw.contiguous(), a_raw.contiguous(), trap_raw.contiguous()
        a.dt_raw, a.a_raw, a.trap_raw = T.ptr(dt_raw), T.ptr(a_raw), T.ptr(trap_raw)
    a.raw_st = T.st_blh(dt_raw)
    a.angles, a.ang_st, a.dt_bias = T.ptr(angles), T.st_bln(angles), T.ptr(dtb)
    a.q_bias, a.k_bias, a.d_skip = T.ptr(qb), T.ptr(kb), T.ptr(dsk)
    a.seed_ssm, a.seed_k, a.seed_v, a.seed_phi = T.ptr(s_ssm), T.ptr(s_k), T.ptr(s_v), T.ptr(s_phi)
    if y is not None:
        a.y, a.y_st = T.ptr(y), T.st_bhlp(y)
    a.final_ssm, a.final_k, a.final_v, a.final_phi = T.ptr(fs), T.ptr(fk), T.ptr(fv), T.ptr(fphi)
    a.kernel = _kernel_code(kernel)
    # head-shared rotary rates, computed once per (b, t, angle) by the tensor-core forward
    wsz = C.lib().m3_siso_fwd_workspace_size(ctypes.byref(a.dims))
    fws, ready = rates if rates is not None else (None, False)
    if fws is None or fws.numel() < wsz:
        fws, ready = torch.empty(wsz, dtype=torch.uint8, device=dev), False
    a.fwd_workspace, a.fwd_workspace_bytes, a.fwd_workspace_ready = T.ptr(fws), wsz, int(bool(ready))
    saved = False
    if bwd_states is not None and C.lib().m3_siso_fwd_saves_states(a):
        a.bwd_states, a.bwd_states_bytes = T.ptr(bwd_states), bwd_states.numel() * bwd_states.element_size()
        saved = True
    C.check(C.lib().m3_siso_fwd(a, T.stream_handle(dev)))
    if return_saved:
        return (y, fs, fk, fv, fphi), saved
    return y, fs, fk, fv, fphi


def final_state_supported(q, v, angles, chunk: int, dtype_policy: str = "bf16") -> bool:
    """Whether `siso_forward_raw(..., states_only=True)` has a kernel for these shapes
    (the tensor-core ones: bf16 I/O and policy, N = 128, P = 64, chunk % 128 == 0)."""
    n, p, nr = q.shape[-1], v.shape[-1], angles.shape[-1]
    return (v.dtype == torch.bfloat16 and T.policy_code(dtype_policy) == C.M3_POLICY_BF16 and n == 128
            and p == 64 and chunk % 128 == 0 and nr % 8 == 0 and nr <= 64 and q.shape[1] % 128 == 0)


_MIN_SEGMENT_CHUNKS = 8  # a segment shorter than this spends more on the extra pass than it gains
_MIN_SEGMENTS = 3  # 2 segments cost 2 x 0.5 x (1 + 0.65) of one pass: no gain
_MAX_SEGMENTS = 64  # m3_siso_split_carry's limit


def _sm_count(device) -> int:
    return torch.cuda.get_device_properties(device).multi_processor_count


def _auto_split(q, v, angles, chunk, dtype_policy, kernel) -> int:
    """Segments per sequence so that B * H * segments sequences fill the SMs once: the
    tensor-core forward runs one sequence per SM at a time.  The split runs a states-only
    pass (~0.65 of a full pass) before the full one, so it pays from 3 segments on."""
    if kernel not in ("auto", "tensorcore") or not final_state_supported(q, v, angles, chunk, dtype_policy):
        return 1
    units = q.shape[0] * v.shape[1]
    nsm = _sm_count(q.device)
    nck = q.shape[1] // chunk
    best = 1
    for g in range(2, min(nck // _MIN_SEGMENT_CHUNKS, _MAX_SEGMENTS) + 1):
        if nck % g == 0 and units * g <= nsm:
            best = g
    return best if best >= _MIN_SEGMENTS else 1


# states-only pass per chunk relative to the full forward is 0.60 standalone; the chain's
# two streams overlap imperfectly, and the cut measured best at about 0.69 of the chunks,
# which this value gives
_ST_COST = 0.55
_MIN_CHAIN_CHUNKS = 16


def _chain_fits(q, v, angles, chunk, dtype_policy, kernel) -> bool:
    """Whether `_forward_raw_chain2` applies: the (b, h) sequences fill at most half the SMs
    (so two passes run side by side) but too many for the length split's equal segments."""
    if kernel not in ("auto", "tensorcore") or not final_state_supported(q, v, angles, chunk, dtype_policy):
        return False
    units = q.shape[0] * v.shape[1]
    return 2 * units <= _sm_count(q.device) and q.shape[1] // chunk >= _MIN_CHAIN_CHUNKS


def _chain_cut(nck: int) -> int:
    """Chunks of the first segment: the full pass of segment 0 (a chunks) ends when the
    states-only pass of segment 0 plus the full pass of segment 1 do, a = _ST_COST a + (nck - a)."""
    return min(nck - 1, max(1, round(nck / (2.0 - _ST_COST))))


_SIDE_STREAMS = {}


def _forward_raw_chain2(q, k, v, dt_raw, a_raw, trap_raw, angles, dt_bias, q_bias, k_bias, d_skip, z,
                        seed_ssm, seed_k, seed_v, seed_phi, a_floor, chunk, dtype_policy, y_out, kernel):
    """The forward of a batch that fills at most half the SMs, as two chained segments of
    unequal length whose passes overlap: on a side stream the full forward of segment 0
    (tokens [0, a)); on the caller's stream the states-only pass of segment 0 (its exact
    final carry, from the caller's carry), then the full forward of segment 1 from that carry
    (the segment chaining of ``siso.py:154-216``).  Both streams hold B * H persistent CTAs,
    so they run side by side; ``a`` balances segment 0's full pass against the states-only
    pass plus segment 1 (`_chain_cut`).  Same results as one pass of the whole sequence."""
    b, l, _ = q.shape
    h, p = v.shape[1], v.shape[3]
    cut = _chain_cut(l // chunk) * chunk
    dev = q.device
    io = v.dtype if v.dtype in (torch.bfloat16, torch.float32) else torch.float32
    if y_out is None:
        y_out = torch.empty(b, h, l, p, dtype=io, device=dev)
    common = dict(d_skip=d_skip, a_floor=a_floor, chunk=chunk, dtype_policy=dtype_policy, kernel=kernel, lsplit=1)
    sl0, sl1 = slice(0, cut), slice(cut, l)
    seg = lambda sl: (q[:, sl], k[:, sl], v[:, :, sl], dt_raw[:, sl], a_raw[:, sl], trap_raw[:, sl], angles[:, sl])
    z0 = None if z is None else z[:, :, sl0]
    z1 = None if z is None else z[:, :, sl1]
    seeds = dict(seed_ssm=seed_ssm, seed_k=seed_k, seed_v=seed_v, seed_phi=seed_phi)
    cur = torch.cuda.current_stream(dev)
    side = _SIDE_STREAMS.get(dev)
    if side is None:
        side = _SIDE_STREAMS[dev] = torch.cuda.Stream(dev)
    side.wait_stream(cur)
    with torch.cuda.stream(side):
        siso_forward_raw(*seg(sl0), dt_bias, q_bias, k_bias, z=z0, y_out=y_out[:, :, sl0], **seeds, **common)
    _, s0, k0, v0, p0 = siso_forward_raw(*seg(sl0), dt_bias, q_bias, k_bias, z=z0, states_only=True, **seeds,
                                         **common)
    _, fs, fk, fv, fphi = siso_forward_raw(*seg(sl1), dt_bias, q_bias, k_bias, z=z1, y_out=y_out[:, :, sl1],
                                           seed_ssm=s0, seed_k=k0, seed_v=v0, seed_phi=p0, **common)
    cur.wait_stream(side)
    return y_out, fs, fk, fv, fphi


def forward_launches(q, v, angles, chunk, dtype_policy="bf16", kernel="auto", lsplit=None) -> int:
    """Kernel launches of one `siso_forward_raw` call with these shapes (no saved states):
    2 for the tensor-core forward (head-shared rotary rates + the scan), 6 when it is split
    over the length (tile sums, entering angles, one rate pass shared by the states-only and
    the full pass, the carry rebuild), 1 for the generic kernel."""
    g = _auto_split(q, v, angles, chunk, dtype_policy, kernel) if lsplit is None else lsplit
    if g > 1:
        return 6
    if lsplit is None and _chain_fits(q, v, angles, chunk, dtype_policy, kernel):
        return 6  # rates + pass for each of the three calls
    tc = kernel in ("auto", "tensorcore", "tensorcore_v1") and final_state_supported(q, v, angles, chunk,
                                                                                       dtype_policy)
    return 2 if tc else 1


def _split_view(t, g):
    """(B, L, ...) -> (B * g, L / g, ...) without a copy when the batch stride is L times the
    token stride (dense or a layer's in_proj slice); else a dense copy first."""
    b, l = t.shape[0], t.shape[1]
    if t.stride(0) != l * t.stride(1):
        t = t.contiguous()
    return t.as_strided((b * g, l // g) + tuple(t.shape[2:]), (t.stride(1) * (l // g),) + tuple(t.stride()[1:]))


def _split_view_bhlp(t, g):
    """(B, H, L, P) -> (B * g, H, L / g, P) (the same rule on the batch and token strides)."""
    b, h, l, p = t.shape
    if t.stride(0) != l * t.stride(2):
        t = t.permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3)
    return t.as_strided((b * g, h, l // g, p), (t.stride(2) * (l // g), t.stride(1), t.stride(2), t.stride(3)))


def _forward_raw_split(q, k, v, dt_raw, a_raw, trap_raw, angles, dt_bias, q_bias, k_bias, d_skip, z,
                       seed_ssm, seed_k, seed_v, seed_phi, a_floor, chunk, dtype_policy, y_out, kernel, g):
    """The forward with every sequence cut into ``g`` segments that run side by side, so a
    batch of few (b, h) sequences still fills the GPU (one sequence per SM at a time).

    Segment j is scanned as if it were chained after segment j-1 (the reference's
    segmentation rule, ``siso.py:154-216``: the carried state plus the trapezoid seed term
    ``dt_0 (1 - lam_0) v_prev k_prev^T``), which equals one scan of the whole sequence.  Its
    entering carry is rebuilt instead of waited for:

    1. the entering angle of every segment: the carry's phi plus the earlier segments' sums
       of tanh(angle) pi dt (tile sums by ``m3_siso_split_prep``, reduced by the angles-only
       ``m3_siso_split_carry``);
    2. pass 1, states only, from a zero state at that angle: each segment's own final state
       S_j, and its true last k and v;
    3. S_end(j) = e^{A_j} (S_end(j-1) + c_j v_{j-1} k_{j-1}^T) + S_j (A_j the segment's sum of
       adt, c_j = dt (1 - lam) of its first token), serially over the segments by the full
       ``m3_siso_split_carry``;
    4. pass 2, the full forward of all segments from their true carries."""
    b, l, n = q.shape
    h, p = v.shape[1], v.shape[3]
    nr = angles.shape[-1]
    if not final_state_supported(q, v, angles, chunk, dtype_policy):
        raise ValueError("lsplit > 1 needs the tensor-core forward (bf16, N = 128, P = 64, chunk % 128 == 0)")
    if g > _MAX_SEGMENTS or l % (chunk * g):
        raise ValueError(f"lsplit = {g}: the chunk count {l // chunk} must split into at most "
                         f"{_MAX_SEGMENTS} equal segments")
    dev, f32 = q.device, torch.float32
    stream = T.stream_handle(dev)
    dt_raw, a_raw, trap_raw, angles = (T.f32c(t) for t in (dt_raw, a_raw, trap_raw, angles))
    if dt_raw.stride() != a_raw.stride() or dt_raw.stride() != trap_raw.stride():
        dt_raw, a_raw, trap_raw = dt_raw.contiguous(), a_raw.contiguous(), trap_raw.contiguous()
    dtb = T.f32dense(dt_bias)
    # 1. per-tile sums of the angle increments and decays, seed coefficients (one kernel)
    tiles = l // (g * C.M3_SPLIT_TILE)
    partial = torch.empty(b, g, tiles, h, nr + 1, dtype=f32, device=dev)
    coef = torch.empty(b, g, h, dtype=f32, device=dev)
    pa = C.M3SplitPrepArgs(b, l, h, nr, g, a_floor, T.ptr(dt_raw), T.ptr(a_raw), T.ptr(trap_raw), T.st_blh(dt_raw),
                           T.ptr(angles), T.st_bln(angles), T.ptr(dtb), T.ptr(partial), T.ptr(coef))
    C.check(C.lib().m3_siso_split_prep(ctypes.byref(pa), stream))
    # views of every (B, L, ...) input as (B * g, L / g, ...)
    qs, ks = _split_view(q, g), _split_view(k, g)
    vs = _split_view_bhlp(v, g)
    zs = None if z is None else _split_view_bhlp(z, g)
    raws = [_split_view(t, g) for t in (dt_raw, a_raw, trap_raw, angles)]
    common = dict(d_skip=d_skip, a_floor=a_floor, chunk=chunk, dtype_policy=dtype_policy, kernel=kernel, lsplit=1)
    seeds = [None if t is None else T.f32dense(t) for t in (seed_ssm, seed_k, seed_v, seed_phi)]
    # 2. segment sums and entering angles; pass 1: each segment's own state from zero at its true angle
    phi_in = torch.empty(b * g, h, nr, dtype=f32, device=dev)
    a_seg = torch.empty(b, g, h, dtype=f32, device=dev)
    ca = C.M3SplitCarryArgs(b, h, g, tiles, n, p, nr, T.ptr(partial), T.ptr(a_seg), T.ptr(coef), None, None, None,
                            *(T.ptr(t) for t in seeds), T.ptr(phi_in), None, None, None)
    C.check(C.lib().m3_siso_split_carry(ctypes.byref(ca), stream))
    # both passes read the same head-shared rotary rates: computed by the first, reused by the second
    d_seg = C.M3Dims(b * g, l // g, h, n, p, nr, chunk)
    rws = torch.empty(C.lib().m3_siso_fwd_workspace_size(ctypes.byref(d_seg)), dtype=torch.uint8, device=dev)
    _, s_loc, k_last, v_last, _ = siso_forward_raw(qs, ks, vs, *raws, dt_bias, q_bias, k_bias, z=zs,
                                                   seed_phi=phi_in, states_only=True, rates=(rws, False),
                                                   **common)
    c_ssm = torch.empty(b * g, h, p, n, dtype=f32, device=dev)
    c_k = torch.empty(b * g, h, n, dtype=f32, device=dev)
    c_v = torch.empty(b * g, h, p, dtype=f32, device=dev)
    ca.c_ssm, ca.c_k, ca.c_v = T.ptr(c_ssm), T.ptr(c_k), T.ptr(c_v)
    # 3. the entering states, k and v of every segment (one kernel, serial over segments)
    ca.s_loc, ca.k_last, ca.v_last = T.ptr(s_loc), T.ptr(k_last), T.ptr(v_last)
    C.check(C.lib().m3_siso_split_carry(ctypes.byref(ca), stream))
    # 4. pass 2: every segment from its true carry (segment 0 without one if the caller had none)
    # (a (B, L, H, P) buffer seen as (B, H, L, P) splits without a copy)
    io = v.dtype if v.dtype in (torch.bfloat16, f32) else f32
    target = y_out
    if y_out is None or y_out.stride(0) != l * y_out.stride(2):
        y_out = torch.empty(b, l, h, p, dtype=io, device=dev).permute(0, 2, 1, 3)
    ys = _split_view_bhlp(y_out, g)
    _, fs, fk, fv, fphi = siso_forward_raw(qs, ks, vs, *raws, dt_bias, q_bias, k_bias, z=zs, seed_ssm=c_ssm,
                                           seed_k=c_k, seed_v=c_v, seed_phi=phi_in, y_out=ys, rates=(rws, True),
                                           **common)
    if target is not None and target.data_ptr() != y_out.data_ptr():
        target.copy_(y_out)
        y_out = target
    last = lambda t: t.unflatten(0, (b, g))[:, g - 1]  # the last segment of every sequence
    return y_out, last(fs), last(fk), last(fv), last(fphi)
