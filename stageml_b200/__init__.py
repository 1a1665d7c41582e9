"""stageml_b200 -- B200 (sm_100a) implementation of StageML's request-time
multi-tenant MoE-LoRA residual path.

The public surface mirrors the reference package ``stageml`` for this path:
``annotations`` (stage0/stage1/compile_staged/BindingTime), ``adapter_bank``,
``adapter_cache``, ``moe_lora_layers``, ``custom_op_registry`` and
``vllm_stage_router``. Their CUDA inputs run on hand-written sm_100a kernels
behind the C ABI in ``include/stageml_b200.h`` (``ops`` is the thin Python
layer over it). Importing the package does not touch CUDA; the native
libraries load on first use of ``stageml_b200.ops``.
"""

from .annotations import BindingTime, compile_staged, stage0, stage1

__version__ = "0.1.0"

__all__ = ["stage0", "stage1", "compile_staged", "BindingTime", "__version__"]
