"""OSCAR INT2 KV-cache hot path for NVIDIA B200 (sm_100a).

Modules mirror the reference plugin's surface: ``config``, ``layout``, ``kernels``,
``calibration_kernels``, ``calibration_worker``, ``calibrate`` (the calibration
driver), ``rotations``, ``metadata``, ``backend``, ``plugin``; ``partition`` splits one
workload over the GPUs of a box by KV head and request.  The device work is in
``liboscar_b200.so`` (C ABI in ``include/oscar_b200.h``), built by
``python -m oscar_new_b200.build``.
"""

__version__ = "0.1.0"
