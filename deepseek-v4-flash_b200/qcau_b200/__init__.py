"""qcau_b200 -- the QCAU path of DeepSeek-V4-Flash on B200 (sm_100a).

Host-side mirror of the reference's interfaces over libqcau_b200.so:

* ``qcau_b200.kernel``  -- act_quant / fp8_gemm / sparse_attn with the
  signatures of Deepseek_origin/inference/kernel.py (install it as
  ``sys.modules["kernel"]`` to run the reference model.py on these kernels);
* ``qcau_b200.QCAU``    -- the QCAU(...) block of
  QCAU/QCAU_inference/inference/QCAU.py;
* ``qcau_b200.mla``     -- the absorbed-MLA decode layer (paged latent cache,
  head sharding with an NCCL all-reduce).

Every call runs the CUDA kernels of the library; there is no CPU path.
"""
from . import _lib, kernel, mla
from .QCAU import QCAU
from ._lib import QcauError, device_error

__all__ = ["QCAU", "kernel", "mla", "device_error", "QcauError"]
