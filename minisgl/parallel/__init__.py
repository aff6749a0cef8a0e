from .comm import (DistributedCommunicator, DistributedImpl, TorchDistributedImpl, destroy_distributed, register_plugin,
                   sequence_parallel_comm)
from .info import (DistributedInfo, get_cp_info, get_dp_info, get_tp_info, reset_cp_info, reset_dp_info, reset_tp_info,
                   set_cp_info, set_dp_info, set_tp_info, try_get_tp_info)

__all__ = [
    "DistributedInfo", "get_tp_info", "set_tp_info", "try_get_tp_info", "reset_tp_info",
    "get_cp_info", "set_cp_info", "reset_cp_info", "get_dp_info", "set_dp_info", "reset_dp_info",
    "DistributedCommunicator", "DistributedImpl", "TorchDistributedImpl", "destroy_distributed",
    "register_plugin", "sequence_parallel_comm",
]
