"""GDNX-B200: sm_100a CUDA kernels for the GDN3 / KMD-2 recurrent-scan hot path.

* ``gdnx_b200.ops``         -- torch-tensor front end of the C ABI (include/gdnx.h)
* ``gdnx_b200.gdn3_upgrade`` -- ``GDN3LinearAttn`` drop-in (``_gdn3_recurrent_state``)
* ``gdnx_b200.kmd2_fast_scan`` -- ``scan`` / ``scan_with_update_norm`` drop-ins
* ``gdnx_b200.distributed`` -- (batch x head) sharding over ranks + output all-gather

The CUDA library ``libgdnx.so`` is built in-tree by ``python -m gdnx_b200.build``;
importing :mod:`gdnx_b200.ops` does not need a GPU, calling it does.
"""
__version__ = "0.1.0"
