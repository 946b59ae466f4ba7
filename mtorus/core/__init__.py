"""L1 core primitives: topology model and FP8 precision (C++ core in ``mtorus._C``)."""
from .coordinator import CollectiveOp, DummyCommunicator, TopologyAwareCommunicator  # noqa: F401
from .precision import (  # noqa: F401
    DelayedScaling, Fp8Format, Fp8Quantizer, Fp8Tensor, LossScaleMode, LossScaler, MasterFormat,
    MixedPrecisionConfig, Quantize, ScalingStrategy, fp8_format_max, from_fp8, to_fp8, to_fp8_per_block,
    to_fp8_with_scale)
from .topology import (  # noqa: F401
    DiscoveryConfig, GPUDevice, IntraNodeMesh, MeshTorusHybrid, TorusCoordinates, TorusDimensions,
    compute_hop_distance, discover_devices, discover_mesh, topology_aware_placement)
