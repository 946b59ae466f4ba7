"""L4 training orchestration: config (TOML), distributed runtime, gradient
accumulator, train_step, device-resident fused optimizers and the end-to-end
GPT trainer."""
from .accumulator import GradientAccumulator, GradientsParams, ParamId, list_param_ids, param_id  # noqa: F401
from .config import PipelineScheduleConfig, TopologyConfig, TrainingConfig, ValidationError  # noqa: F401
from .runtime import (DistributedRuntime, DistributedRuntimeBuilder, DistributedRuntimeError,  # noqa: F401
                      init_distributed, loss_scaler_from_config)
from .step import (Counter, StepError, StepMetrics, TrainingError, TrainingMetrics, apply_clip_norm,  # noqa: F401
                   check_overflow_values, clip_grad_norm, compute_grad_norm, train_step, training_loop)
