"""flash_aurora_b200: the Aurora Swin3D backbone block hot path on NVIDIA B200 (sm_100a).

Hand-written CUDA kernels behind a C ABI (``include/flash_aurora_b200.h``,
``libflash_aurora_b200.so`` built in-tree by ``python -m flash_aurora_b200.build``), with a
PyTorch host layer that mirrors the operator interface of upstream Flash-Aurora:

* ``swin3d_layout``  roll_pad_partition_windows / crop_roll_unmerge_windows
                     (upstream ``ops/triton_swin3d_layout.py``)
* ``adaln``          adaptive_layernorm_film_forward / ..._add_residual_forward
                     (upstream ``ops/triton_adaln.py``)
* ``window_attn``    WinAttnPrecision, window_attn_fwd_cute, window_attn_fwd_cute_qkvpacked,
                     window_attn_dispatch (upstream ``ops/cute/window_attn_fwd.py``)
* ``swin3d``         Swin3DTransformerBlock / Swin3DTransformerBackbone with upstream state-dict
                     keys (upstream ``aurora/model/swin3d.py``, ``film.py``)
* ``sharding``       latitude-band window sharding with a point-to-point halo exchange
* ``custom_op_paths`` can_use_* gating predicates (upstream ``aurora/model/custom_op_paths.py``)
* ``status``         device-side failure status of the pipelined kernels, checked on the host
"""

from .activation import gelu_erf
from .linear import linear_bias_act
from .perceiver_ln import layernorm_affine_add_residual_forward, layernorm_affine_forward
from .adaln import (
    adaptive_layernorm_film_add_residual_forward,
    adaptive_layernorm_film_add_residual_rows,
    adaptive_layernorm_film_forward,
    unmerge_adaptive_layernorm_film_add_residual,
    unmerge_adaptive_layernorm_film_add_residual_band,
)
from .sharding import BandContext, HaloExchangeError, band_bounds
from .swin3d_layout import (
    band_halo_extract,
    crop_roll_unmerge_windows,
    crop_roll_unmerge_windows_band,
    crop_roll_unmerge_windows_triton,
    roll_pad_partition_windows,
    roll_pad_partition_windows_band,
    roll_pad_partition_windows_triton,
)
from .util import band_geometry, maybe_adjust_windows, window_geometry
from .window_attn import (
    WinAttnPrecision,
    shifted_window_group_ids,
    window_attn_dispatch,
    window_attn_fwd_cute,
    window_attn_fwd_cute_qkvpacked,
)
from .workspace_pool import InferenceWorkspacePool
from .status import DeviceStatusError, check_device_status, device_status, reset_device_status, watchdog_selftest
from .custom_op_paths import (
    can_use_cute_qkvpacked,
    can_use_cute_window_attention,
    can_use_triton_adaln,
    can_use_triton_gelu,
    can_use_triton_layout,
)

__all__ = [
    "gelu_erf",
    "linear_bias_act",
    "layernorm_affine_forward",
    "layernorm_affine_add_residual_forward",
    "adaptive_layernorm_film_add_residual_forward",
    "adaptive_layernorm_film_add_residual_rows",
    "adaptive_layernorm_film_forward",
    "unmerge_adaptive_layernorm_film_add_residual",
    "unmerge_adaptive_layernorm_film_add_residual_band",
    "BandContext",
    "HaloExchangeError",
    "band_bounds",
    "band_geometry",
    "band_halo_extract",
    "crop_roll_unmerge_windows_band",
    "roll_pad_partition_windows_band",
    "crop_roll_unmerge_windows",
    "crop_roll_unmerge_windows_triton",
    "roll_pad_partition_windows",
    "roll_pad_partition_windows_triton",
    "maybe_adjust_windows",
    "window_geometry",
    "WinAttnPrecision",
    "shifted_window_group_ids",
    "window_attn_dispatch",
    "window_attn_fwd_cute",
    "window_attn_fwd_cute_qkvpacked",
    "InferenceWorkspacePool",
    "DeviceStatusError",
    "check_device_status",
    "device_status",
    "reset_device_status",
    "watchdog_selftest",
    "can_use_cute_qkvpacked",
    "can_use_cute_window_attention",
    "can_use_triton_adaln",
    "can_use_triton_gelu",
    "can_use_triton_layout",
]
