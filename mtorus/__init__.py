"""mtorus: a Blackwell-native mesh-torus distributed training framework.

Layers (bottom-up): ``core`` (topology, FP8 precision), ``comm`` (communicators),
``pipeline`` (stages, schedules, executors), ``torch_ext`` (FP8 <-> torch glue),
``training`` (config, runtime, accumulator, train_step, fused trainer),
``models`` (GPT), ``ops`` (sm_100a kernels), ``parallel`` (flat buffers, DP,
peer-memory collectives), ``utils``.
"""
__version__ = "0.1.0"
