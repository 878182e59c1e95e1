"""B200-native (sm_100a) quaternion linear layer.

Drop-in for the hot path of the reference's ``quaternion`` package: the
Hamilton-product layer ``QuaternionLinear`` (``quaternion/linear.py``), its
K1/K2 operator entry points (``quaternion/planar.py``), the LoRA residual
(``quaternion/lora.py``), the packing convention (``quaternion/packing.py``)
and the ``kernels/`` operator interface.  Every quaternion product runs in the
in-tree CUDA library ``lib/libqlin_b200.so`` (C ABI in ``include/qlin_b200.h``):
a TMA + tcgen05/TMEM tensor-core kernel for bf16/f16 and a CUDA-core kernel
for fp32.  There is no CPU path; CPU tensors raise ``RuntimeError``.

The directory name is not a Python identifier, so import it with
``importlib.import_module("quaternion-based-math-1_b200")``.
"""

from . import ops
from .convert import ConversionRecord, convert_model, eligible_modules, project_onto_quaternion
from ._lib import device_error
from .linear import QuaternionLinear, fused_quaternion_linear, pack_quaternion_weights, quaternion_linear
from .lora import (
    LoRAQuaternionLinear,
    count_trainable,
    inject_lora,
    lora_parameters,
    mark_only_lora_trainable,
)
from .packing import (
    build_block_matrix,
    check_divisible,
    pack_components,
    pack_real_to_quaternion,
    split_components,
    unpack_quaternion_to_real,
)
from .planar import planar_coefficient_tensor, quaternion_linear_naive, quaternion_linear_planar
from .reparam import FactorizedQuaternionLinear, UnitQuaternionLinear, normalize_quaternion, parameter_count
from .sharded import ColumnParallelQuaternionLinear, MulticastOutputs, PeerOutputs, gather_columns, shard_bounds

__all__ = [
    "QuaternionLinear",
    "quaternion_linear",
    "fused_quaternion_linear",
    "pack_quaternion_weights",
    "quaternion_linear_naive",
    "quaternion_linear_planar",
    "planar_coefficient_tensor",
    "LoRAQuaternionLinear",
    "inject_lora",
    "lora_parameters",
    "mark_only_lora_trainable",
    "count_trainable",
    "pack_real_to_quaternion",
    "unpack_quaternion_to_real",
    "split_components",
    "pack_components",
    "build_block_matrix",
    "check_divisible",
    "FactorizedQuaternionLinear",
    "parameter_count",
    "UnitQuaternionLinear",
    "normalize_quaternion",
    "convert_model",
    "eligible_modules",
    "project_onto_quaternion",
    "ConversionRecord",
    "ColumnParallelQuaternionLinear",
    "PeerOutputs",
    "MulticastOutputs",
    "gather_columns",
    "shard_bounds",
    "device_error",
    "ops",
]
