"""CPU checks of the C ABI: the library loads, exports every entry point the header
declares, the ctypes structs match the C layout, and argument validation rejects bad
calls with the documented codes before anything reaches a GPU."""

import ctypes
import os
import re
import subprocess
import tempfile

import pytest

from mamba3_b200 import _capi as C

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "m3_siso.h")


def _declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(m3_\w+)\s*\(", src, re.M)))


def test_library_exports_every_declared_symbol():
    lib = C.lib()
    names = _declared()
    assert set(names) == set(C.EXPORTS)
    for n in names:
        assert hasattr(lib, n), n
    assert lib.m3_version() >= 1


def test_struct_layout_matches_header():
    prog = r'''
#include <stdio.h>
#include <stddef.h>
#include "m3_siso.h"
int main(void) {
  printf("%zu %zu %zu %zu %zu\n", sizeof(M3Dims), sizeof(M3Strides), sizeof(M3FwdArgs),
         sizeof(M3BwdArgs), sizeof(M3DecodeArgs));
  printf("%zu %zu %zu %zu\n", offsetof(M3FwdArgs, chunk_states_dtype), offsetof(M3BwdArgs, workspace_bytes),
         offsetof(M3DecodeArgs, y), offsetof(M3FwdArgs, fwd_workspace_ready));
  printf("%zu %zu %zu %zu\n", sizeof(M3SampleArgs), offsetof(M3SampleArgs, seed), offsetof(M3SampleArgs, stop_ids),
         offsetof(M3SampleArgs, probs_ld));
  printf("%zu %zu %zu %zu\n", sizeof(M3SplitPrepArgs), offsetof(M3SplitPrepArgs, coef), sizeof(M3SplitCarryArgs),
         offsetof(M3SplitCarryArgs, c_v));
  printf("%zu %zu %zu %zu\n", sizeof(M3GemvArgs), offsetof(M3GemvArgs, tickets), sizeof(M3GemmArgs),
         offsetof(M3GemmArgs, ldo));
  return 0;
}
'''
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        exe = os.path.join(d, "t")
        open(c, "w").write(prog)
        subprocess.check_call(["gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe])
        out = subprocess.check_output([exe]).decode().split()
    got = [int(x) for x in out]
    want = [ctypes.sizeof(C.M3Dims), ctypes.sizeof(C.M3Strides), ctypes.sizeof(C.M3FwdArgs),
            ctypes.sizeof(C.M3BwdArgs), ctypes.sizeof(C.M3DecodeArgs),
            C.M3FwdArgs.chunk_states_dtype.offset, C.M3BwdArgs.workspace_bytes.offset, C.M3DecodeArgs.y.offset,
            C.M3FwdArgs.fwd_workspace_ready.offset,
            ctypes.sizeof(C.M3SampleArgs), C.M3SampleArgs.seed.offset, C.M3SampleArgs.stop_ids.offset,
            C.M3SampleArgs.probs_ld.offset,
            ctypes.sizeof(C.M3SplitPrepArgs), C.M3SplitPrepArgs.coef.offset, ctypes.sizeof(C.M3SplitCarryArgs),
            C.M3SplitCarryArgs.c_v.offset,
            ctypes.sizeof(C.M3GemvArgs), C.M3GemvArgs.tickets.offset, ctypes.sizeof(C.M3GemmArgs),
            C.M3GemmArgs.ldo.offset]
    assert got == want


def _fwd(**kw):
    a = C.M3FwdArgs()
    a.dims = C.M3Dims(2, 128, 3, 128, 64, 32, 64)
    a.io_dtype, a.policy, a.raw = C.M3_DTYPE_F32, C.M3_POLICY_F32, 0
    fake = 256
    for f in ("q", "k", "v", "adt", "gamma", "scale", "phi", "q_bias", "k_bias", "y", "final_ssm",
              "final_k", "final_v"):
        setattr(a, f, fake)
    for k, v in kw.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("mut,code,frag", [
    (dict(dims=C.M3Dims(2, 128, 3, 128, 64, 32, 96)), C.M3_ERR_UNSUPPORTED, "chunk"),
    (dict(dims=C.M3Dims(2, 100, 3, 128, 64, 32, 64)), C.M3_ERR_SHAPE, "multiple of chunk"),
    (dict(dims=C.M3Dims(2, 128, 3, 128, 64, 80, 64)), C.M3_ERR_SHAPE, "n_angles"),
    (dict(dims=C.M3Dims(2, 128, 3, 96, 64, 32, 64)), C.M3_ERR_UNSUPPORTED, "state_dim"),
    (dict(dims=C.M3Dims(0, 128, 3, 128, 64, 32, 64)), C.M3_ERR_SHAPE, "positive"),
    (dict(q=None), C.M3_ERR_ARG, "required"),
    (dict(adt=None), C.M3_ERR_ARG, "preprocessed"),
    (dict(seed_ssm=256), C.M3_ERR_ARG, "together"),
    (dict(io_dtype=7), C.M3_ERR_ARG, "io_dtype"),
    (dict(raw=1), C.M3_ERR_ARG, "raw boundary"),
    (dict(y=None), C.M3_ERR_UNSUPPORTED, "final state only"),  # f32 I/O has no states-only kernel
])
def test_fwd_validation_errors(mut, code, frag):
    a = _fwd(**mut)
    rc = C.lib().m3_siso_fwd(a, None)
    assert rc == code
    assert frag in C.lib().m3_last_error().decode()


def test_bwd_workspace_validation():
    a = C.M3BwdArgs()
    a.dims = C.M3Dims(1, 128, 2, 32, 32, 8, 64)
    for f in ("q", "k", "v", "adt", "gamma", "scale", "phi", "q_bias", "k_bias", "dy", "dq", "dk", "dv",
              "dq_bias", "dk_bias", "dadt", "dgamma", "dscale", "dphi"):
        setattr(a, f, 256)
    need = C.lib().m3_siso_bwd_workspace_size(ctypes.byref(a.dims))
    assert need >= 1 * 2 * (128 // 32) * 32 * 32 * 4
    a.workspace, a.workspace_bytes = 256, need - 1
    assert C.lib().m3_siso_bwd(a, None) == C.M3_ERR_WORKSPACE


def test_decode_validation():
    a = C.M3DecodeArgs()
    a.batch, a.nheads, a.state_dim, a.headdim, a.n_angles = 2, 2, 48, 16, 4
    assert C.lib().m3_siso_decode(a, None) == C.M3_ERR_UNSUPPORTED
    a.state_dim = 32
    assert C.lib().m3_siso_decode(a, None) == C.M3_ERR_ARG


def test_sample_validation():
    """Argument checks of m3_sample_tokens run on the host, before any launch."""
    a = C.M3SampleArgs()
    assert C.lib().m3_sample_tokens(a, None) == C.M3_ERR_ARG  # no logits / output
    a.logits, a.out_token = 16, 16  # never dereferenced: validation fails first
    a.batch, a.vocab, a.logits_ld = 1, 100, 50
    assert C.lib().m3_sample_tokens(a, None) == C.M3_ERR_SHAPE  # leading dimension < vocab
    a.logits_ld, a.logits_dtype = 100, 7
    assert C.lib().m3_sample_tokens(a, None) == C.M3_ERR_UNSUPPORTED
    a.logits_dtype, a.temperature, a.rep_penalty, a.top_p = C.M3_DTYPE_F32, 0.0, 1.0, 0.9
    assert C.lib().m3_sample_tokens(a, None) == C.M3_ERR_ARG  # temperature must be > 0
    a.temperature, a.window, a.rep_window = 1.0, 16, 0
    assert C.lib().m3_sample_tokens(a, None) == C.M3_ERR_ARG  # window without its state
    a.window, a.history = None, 16
    assert C.lib().m3_sample_tokens(a, None) == C.M3_ERR_ARG  # history without a counter
    a.history, a.batch = None, 0
    assert C.lib().m3_sample_tokens(a, None) == C.M3_OK  # nothing to do


def test_jax_ffi_shim_binds_only_exported_entry_points():
    """The jax.ffi handlers (``jax_ffi/m3_ffi.cc``) cannot be built here (no jaxlib / XLA FFI
    headers); check that every library call they make is an entry point of the C ABI, and
    that the Python side refuses to import without JAX instead of failing later."""
    import importlib
    import re

    src = open(os.path.join(ROOT, "mamba3-siso-tpu_b200", "jax_ffi", "m3_ffi.cc")).read()
    header = open(os.path.join(ROOT, "include", "m3_siso.h")).read()
    calls = set(re.findall(r"\b(m3_[a-z0-9_]+)\(", src))
    assert calls >= {"m3_siso_fwd", "m3_siso_bwd_noalloc", "m3_siso_decode", "m3_last_error"}
    for c in calls:
        assert re.search(rf"\b{c}\s*\(", header), c
    try:
        import jax  # noqa: F401
    except ImportError:
        with pytest.raises(ImportError):
            importlib.import_module("jax_ffi")
