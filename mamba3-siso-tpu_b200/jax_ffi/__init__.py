"""jax.ffi registration of the B200 kernels (``m3_ffi.cc`` built into ``libm3ffi.so``).

The drop-in for JAX callers of the reference: ``siso_forward``, ``siso_backward`` and
``decode_step`` with the signatures of ``mamba3_pallas/kernel_fwd.py:204``,
``kernel_bwd.py:534`` and ``kernel_decode.py:467``, each one XLA custom call on the CUDA
platform instead of a ``pallas_call``.  JAX is not installed with this repository; importing
this module without it raises ImportError, and nothing else in the package imports it.
"""

from __future__ import annotations

import ctypes
import os

import jax  # noqa: F401  (ImportError when JAX is absent: this module is optional)
import jax.numpy as jnp

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = os.environ.get("M3_FFI_LIB", os.path.join(_HERE, "libm3ffi.so"))
_POLICY = {"f32": 0, "bf16": 1}
_registered = False


def register():
    """Load ``libm3ffi.so`` (and through it libm3siso.so) and register the three targets."""
    global _registered
    if _registered:
        return
    lib = ctypes.CDLL(_LIB)
    for name, sym in (("m3_siso_fwd", "kM3SisoFwd"), ("m3_siso_bwd", "kM3SisoBwd"),
                      ("m3_siso_decode", "kM3SisoDecode")):
        jax.ffi.register_ffi_target(name, jax.ffi.pycapsule(getattr(lib, sym)), platform="CUDA")
    _registered = True


def siso_forward(q, k, v, adt, gamma, scale, phi, q_bias, k_bias, d_skip, z, chunk=128, dtype_policy="bf16"):
    """``kernel_fwd.siso_forward``: returns ``(y, final_ssm, final_k, final_v)``."""
    register()
    B, L, N = q.shape
    H, P = v.shape[1], v.shape[3]
    outs = (jax.ShapeDtypeStruct(v.shape, v.dtype), jax.ShapeDtypeStruct((B, H, P, N), jnp.float32),
            jax.ShapeDtypeStruct((B, H, N), jnp.float32), jax.ShapeDtypeStruct((B, H, P), jnp.float32))
    return jax.ffi.ffi_call("m3_siso_fwd", outs)(q, k, v, z, adt, gamma, scale, phi, q_bias, k_bias, d_skip,
                                                 chunk=jnp.int32(chunk), policy=jnp.int32(_POLICY[dtype_policy]))


def siso_backward(dy, q, k, v, adt, gamma, scale, phi, q_bias, k_bias, d_skip, z, chunk=128, dtype_policy="bf16"):
    """``kernel_bwd.siso_backward`` (no seeds): the gradients of q, k, v, z, adt, gamma,
    scale, phi, q_bias, k_bias, d_skip, all float32."""
    register()
    f = lambda t: jax.ShapeDtypeStruct(t.shape, jnp.float32)
    outs = tuple(f(t) for t in (q, k, v, z, adt, gamma, scale, phi, q_bias, k_bias, d_skip))
    return jax.ffi.ffi_call("m3_siso_bwd", outs)(dy, q, k, v, z, adt, gamma, scale, phi, q_bias, k_bias, d_skip,
                                                 chunk=jnp.int32(chunk), policy=jnp.int32(_POLICY[dtype_policy]))


def decode_step(q, k, v, adt, dt, lam, angles, q_bias, k_bias, state, d_skip, z, dtype_policy="bf16"):
    """``kernel_decode.decode_step``: returns ``(y, (ssm, k, v, phi))``; the state buffers are
    donated to the call and updated in place."""
    register()
    ssm, sk, sv, sphi = state
    outs = (jax.ShapeDtypeStruct(v.shape, v.dtype), jax.ShapeDtypeStruct(ssm.shape, jnp.float32),
            jax.ShapeDtypeStruct(sk.shape, jnp.float32), jax.ShapeDtypeStruct(sv.shape, jnp.float32),
            jax.ShapeDtypeStruct(sphi.shape, jnp.float32))
    call = jax.ffi.ffi_call("m3_siso_decode", outs, input_output_aliases={11: 1, 12: 2, 13: 3, 14: 4})
    y, *st = call(q, k, v, z, adt, dt, lam, angles, q_bias, k_bias, d_skip, ssm, sk, sv, sphi,
                  policy=jnp.int32(_POLICY[dtype_policy]))
    return y, tuple(st)
