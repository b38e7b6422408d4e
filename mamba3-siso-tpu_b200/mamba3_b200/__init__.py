"""B200-native Mamba-3 SISO scan: a drop-in for the kernel path of mamba3_pallas.

Module map (reference module -> this package):
  kernel_fwd.siso_forward       -> kernel_fwd.siso_forward / siso_forward_raw
  kernel_bwd.siso_backward      -> kernel_bwd.siso_backward / siso_backward_raw
  kernel_decode.decode_step     -> kernel_decode.decode_step / siso_decode_raw
  siso.siso / siso_segment      -> siso.siso / siso_segment
  layer, model, train           -> layer, model, train
  reference.SISOState etc.      -> state
Every compute call goes through libm3siso.so (``_lib/``); there is no CPU path.
"""

from . import checkpoint, convert, layout, state  # noqa: F401
from .layer import SISOConfig, SISOParams, init_params, mamba3_siso_layer, rms_norm, split_in_proj  # noqa: F401
from .model import LMConfig, init_lm, lm_decode_step, lm_forward, zero_states  # noqa: F401
from .siso import SISOOutput, siso_segment, siso_segment_seq_parallel, siso_segment_streamed  # noqa: F401
from .state import SISOState, zero_state  # noqa: F401

__version__ = "0.1.0"
