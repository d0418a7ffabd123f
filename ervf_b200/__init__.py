"""ervf_b200 -- B200-native (sm_100a) NVFP4 expert-GEMV path of kennydd001/ervf.

The compute lives in ``libervf_b200.so`` (C ABI: ``include/ervf_b200.h``),
built by ``python -m ervf_b200.build``.  Python front ends:

  * ``FusedNVFP4``   -- drop-in for lightningstream_nemotron.fused_nvfp4.FusedNVFP4
  * ``GPUKernels``   -- ``mv_bf16`` of lightningstream_nemotron.gpu_kernels
  * ``ExpertBank``   -- HBM-resident expert storage (residency / upload path)
  * ``MoEDecoder``   -- routed-expert MoE layers and decode steps on the C ABI
"""

from .fused_nvfp4 import FusedNVFP4  # noqa: F401
from .gpu_kernels import GPUKernels  # noqa: F401

__version__ = "0.1.0"
