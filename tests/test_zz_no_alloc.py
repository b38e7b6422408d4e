"""m3_siso_bwd_noalloc: the backward for callers that cannot allocate device memory.

Such callers (a custom call or plugin handed only its inputs and outputs by an allocator
it does not own, or a server that forbids device allocation after start-up) get the
same gradients as from m3_siso_bwd, with the scratch taken from a fixed array inside the
library instead of a caller-allocated workspace.  This file checks, through the C ABI,
that two consecutive calls (different inputs, so the second sees the first's leftover
scratch) each match m3_siso_bwd within the parity tolerance, and that a problem too
large for the built-in scratch is refused.  It is collected last on purpose.
"""

import ctypes

import pytest
import torch

from tests.inputs import make_inputs
from tests.metrics import rel_error

pytestmark = pytest.mark.gpu

B, H, L, N, P, NR, CHUNK = 2, 3, 256, 128, 64, 32, 128


def _lib():
    from mamba3_b200 import _capi as C

    lib = C.lib()
    lib.m3_siso_bwd_noalloc.argtypes = [ctypes.POINTER(C.M3BwdArgs), ctypes.c_void_p]
    lib.m3_siso_bwd_noalloc.restype = ctypes.c_int
    lib.m3_siso_bwd_noalloc_scratch_bytes.argtypes = []
    lib.m3_siso_bwd_noalloc_scratch_bytes.restype = ctypes.c_size_t
    return C, lib


def _case(seed):
    x = make_inputs(B, H, L, state_dim=N, headdim=P, n_angles=NR, seed=seed)
    x["dt_bias"] = torch.randn(H, dtype=torch.float64, generator=torch.Generator().manual_seed(seed)) * 0.3
    return {k: v.to("cuda", torch.float32).contiguous() for k, v in x.items()}


def _args(C, d):
    """Raw-boundary backward arguments; outputs are fresh tensors owned by the caller."""
    f = torch.float32
    out = {
        "dq": torch.empty(B, L, N, dtype=f, device="cuda"), "dk": torch.empty(B, L, N, dtype=f, device="cuda"),
        "dv": torch.empty(B, H, L, P, dtype=f, device="cuda"), "dz": torch.empty(B, H, L, P, dtype=f, device="cuda"),
        "ddt_raw": torch.empty(B, L, H, dtype=f, device="cuda"), "da_raw": torch.empty(B, L, H, dtype=f, device="cuda"),
        "dtrap_raw": torch.empty(B, L, H, dtype=f, device="cuda"),
        "dangles": torch.empty(B, L, NR, dtype=f, device="cuda"), "ddt_bias": torch.empty(H, dtype=f, device="cuda"),
        "dq_bias": torch.empty(H, N, dtype=f, device="cuda"), "dk_bias": torch.empty(H, N, dtype=f, device="cuda"),
        "dd_skip": torch.empty(H, dtype=f, device="cuda"),
    }
    a = C.M3BwdArgs()
    a.dims = C.M3Dims(B, L, H, N, P, NR, CHUNK)
    a.io_dtype, a.policy, a.raw, a.a_floor = C.M3_DTYPE_F32, C.M3_POLICY_F32, 1, 1e-4
    for name in ("q", "k", "v", "z", "dt_raw", "a_raw", "trap_raw", "angles", "dt_bias", "q_bias", "k_bias",
                 "d_skip", "dy"):
        setattr(a, name, d[name].data_ptr())
    for name, t in out.items():
        setattr(a, name, t.data_ptr())
    return a, out


def _reference_grads(C, lib, d):
    a, out = _args(C, d)
    ws = torch.empty(lib.m3_siso_bwd_workspace_size(ctypes.byref(a.dims)), dtype=torch.uint8, device="cuda")
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    assert lib.m3_siso_bwd(a, torch.cuda.current_stream().cuda_stream) == C.M3_OK, lib.m3_last_error()
    torch.cuda.synchronize()
    return out


def test_noalloc_backward_matches_allocating_entry_point_twice():
    C, lib = _lib()
    dims = C.M3Dims(B, L, H, N, P, NR, CHUNK)
    assert lib.m3_siso_bwd_workspace_size(ctypes.byref(dims)) <= lib.m3_siso_bwd_noalloc_scratch_bytes()
    stream = torch.cuda.current_stream().cuda_stream
    for seed in (101, 202):  # two calls in a row; the second reuses the first's scratch
        d = _case(seed)
        want = _reference_grads(C, lib, d)
        a, got = _args(C, d)
        a.workspace, a.workspace_bytes = None, 0  # ignored by the no-alloc entry point
        rc = lib.m3_siso_bwd_noalloc(a, stream)
        assert rc == C.M3_OK, lib.m3_last_error()
        torch.cuda.synchronize()
        for name in want:
            e = rel_error(got[name], want[name])
            assert e < 1e-5, (seed, name, e)


def test_noalloc_rejects_problems_beyond_the_scratch():
    C, lib = _lib()
    a = C.M3BwdArgs()
    a.dims = C.M3Dims(64, 8192, 32, 128, 64, 64, 128)  # ~2 GiB of chunk states
    assert lib.m3_siso_bwd_workspace_size(ctypes.byref(a.dims)) > lib.m3_siso_bwd_noalloc_scratch_bytes()
    assert lib.m3_siso_bwd_noalloc(a, None) == C.M3_ERR_WORKSPACE
    assert b"scratch" in lib.m3_last_error()
