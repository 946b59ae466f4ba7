"""L3 pipeline parallelism: stages, FP8 stage transfer, GPipe / 1F1B schedules,
executors (simulated and multi-rank), activation checkpointing, placement."""
from .checkpoint import ActivationCheckpoint, CheckpointHandle, CheckpointStrategy, apply_checkpoint_forward  # noqa: F401
from .communicator import PipelineComm  # noqa: F401
from .executor import DistributedPipelineExecutor, PipelineConfig, PipelineExecutor  # noqa: F401
from .placement import compute_hop_distance, topology_aware_placement  # noqa: F401
from .schedule import (GpipeSchedule, OneF1BSchedule, PipeOp, Schedule, ScheduleKind, ScheduleType,  # noqa: F401
                       build_schedule, ideal_bubble_fraction, rank_program, simulate_schedule)
from .stage import PipelineStage, StageData, StageForward, StageForwardClosure  # noqa: F401
