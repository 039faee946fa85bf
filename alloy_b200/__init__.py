"""alloy_b200: B200 (sm_100a) kernels for the Mamba-2 mixer hot path of gxcsoccer/alloy.

* ``alloy_b200.mixer``        functional API (conv1d+SiLU, fused SSD prefill,
                              pre-discretised scan, decode step)
* ``alloy_b200.kernels``      drop-in names of alloy/models/mamba_kernels.py
* ``alloy_b200.mamba_block``  ``MambaBlock`` / ``MambaCache`` with the
                              reference's signatures
* ``alloy_b200.sharding``     (batch, head-group) partitioning across GPUs
* ``alloy_b200.mlx_bridge``   MLX arrays in and out (DLPack / numpy)

All compute runs in ``liballoy_ssd.so`` (C ABI: include/alloy_ssd.h).
"""

from ._lib import AlloyError, AlloyLibraryError, load as load_library  # noqa: F401

__version__ = "0.1.0"
