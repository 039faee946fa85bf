"""CPU oracle for the Mamba-2 mixer hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the algorithm of gxcsoccer/alloy's Mamba-2
mixer (``alloy/models/mamba_block.py`` and ``alloy/models/mamba_kernels.py``)
so that the CUDA kernels of ``alloy_b200`` can be checked against it.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it, and only as the
checker or the timed CPU baseline.  The product path (``alloy_b200``) never
imports it and has no CPU fallback.

Pinning: MLX (``mlx>=0.22.0``, un-pinned in the reference's pyproject.toml:29)
cannot be installed here, so MLX's own arithmetic is not reproduced bit for
bit.  The oracle is pinned against golden vectors made by executing the
reference's own ``mamba_block.py`` / ``cache.py`` source over a numpy stand-in
for the elementary MLX ops they call (``tests/golden/make_golden.py``), and
against the invariants the reference's tests hold (conv kernel == conv ops,
chunked scan == sequential scan, chunked prefill == step-by-step decode).
"""

from .mamba_ref import *  # noqa: F401,F403
