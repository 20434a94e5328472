"""vxmoe: the routed sparse-MoE block of Veystrix Flash-Next on NVIDIA B200.

Python host layer over libvxmoe.so (hand-written sm_100a CUDA behind the C
ABI of include/vxmoe.h).  Public surfaces follow the reference:

* ``gather_qmm`` / ``quantized_matmul`` - the MLX operators
  (models/flashnext/expert_cache.py:818-829);
* ``build_executor`` / ``MoEExecutor.execute`` - the executor plugin
  (metal_runtime.py:427-983; tests/bench/bench_runtime_layer.py:85-201);
* ``SwitchGLU`` / ``MoEBlock`` / ``moe_call`` - the block
  (expert_cache.py:1709-1772; adaptive_topk.py:54-293).
"""
from .ops import (  # noqa: F401
    GROUP_SIZE, BITS, MoEWeights, Q4Projection, dequantize, gather_qmm, moe_block, moe_experts,
    GraphedBlock, moe_experts_partial, permute, quantized_matmul, rms_norm, route, router, softmax_topk,
    swiglu,
)
from .executor import (  # noqa: F401
    MoEExecutor, Executor, build_executor, create_executor, probe_capabilities, weighted_combine,
    Q4G32Projection,
)
from .block import MoEBlock, SwitchGLU, moe_call  # noqa: F401
from .residency import SlotAssigner, SlotPool  # noqa: F401

__version__ = "0.1.0"
