"""B200-native engine behind Cascade-LLM's ``layer_streaming`` API.

Re-exports the same names as the reference package
(``layer_streaming/__init__.py:3-45``) so that callers such as
``tools/run_llama31.py`` run unchanged; the compute underneath is the
sm_100a kernel library ``libcascade_b200.so`` (see :mod:`.ops`).
"""

from .llama31 import (
    LLAMA31_8B_MODEL_ID,
    DecodeState,
    Llama31DecodeExecutor,
    SimpleKVCache,
    StaticKVCache,
)
from .plan import (
    Granularity,
    HostPlacement,
    ModelPlan,
    TensorSpec,
    TransferUnit,
    VocabPlan,
    build_llama31_8b_plan,
)
from .runtime import DoubleBufferRuntime, HBMResidentRuntime, ResidentDeviceArena
from .vocab import VocabStreamingRuntime, merge_topk
from .weight_store import (
    FullPinnedWeightStore,
    PinnedStagingWeightStore,
    WeightStoreMode,
    create_weight_store,
)

__all__ = [
    "DoubleBufferRuntime",
    "FullPinnedWeightStore",
    "Granularity",
    "HostPlacement",
    "LLAMA31_8B_MODEL_ID",
    "Llama31DecodeExecutor",
    "ModelPlan",
    "PinnedStagingWeightStore",
    "ResidentDeviceArena",
    "SimpleKVCache",
    "TensorSpec",
    "TransferUnit",
    "VocabPlan",
    "VocabStreamingRuntime",
    "WeightStoreMode",
    "build_llama31_8b_plan",
    "create_weight_store",
    "merge_topk",
    # additions of this engine
    "DecodeState",
    "HBMResidentRuntime",
    "StaticKVCache",
]
