"""L2 communication: the Communicator interface and its backends (mock, in-process
threads, P2P channels, TCP, torch.distributed/NCCL, and the device backend over
NVLink peer memory, ``SymmCommunicator``) and the topology-aware wrapper.  The
bandwidth kernels behind the device backend live in ``mtorus.parallel.symm``."""
from .base import CommError, CommTimeout, Communicator, DType, FaultPlan, FaultRule, ReduceOp, from_u64, u64  # noqa: F401
from .local import LocalCommunicator, local_world, run_threads  # noqa: F401
from .mock import MockCommunicator  # noqa: F401
from .p2p import AsyncP2PChannel, P2PChannel, P2PHandle  # noqa: F401
from .tcp import TcpCommunicator, recv_frame, send_frame  # noqa: F401
from .topology_aware import TopologyAwareComm  # noqa: F401
from .device import SymmCommunicator  # noqa: F401,E402
