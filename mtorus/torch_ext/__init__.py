"""L3' framework glue: FP8 <-> torch conversions, autograd FP8 casts, module
splitting into pipeline stages, FP8-gradient optimizers."""
from .autodiff_ext import AutodiffExt, Fp8CastFn, GradientHook, fp8_cast, gradient_cast_e5m2, weight_cast_e4m3  # noqa: F401
from .fp8_ops import (DeviceFp8Tensor, dequantize_tensor, fp8_to_torch, fp8_to_torch_1d, fp8_to_torch_2d,  # noqa: F401
                      quantize_tensor, torch_1d_to_fp8, torch_2d_to_fp8, torch_to_fp8)
from .module_ext import PipelineModule, PipelineStage, SequentialStages, StageForward, split_evenly  # noqa: F401
from .optim_ext import Fp8Adam, Fp8Gradients, Fp8Optimizer, Fp8Sgd, cast_from_fp8, cast_to_fp8, update_weight_fp8  # noqa: F401
