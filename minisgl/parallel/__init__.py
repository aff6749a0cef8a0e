from .comm import DistributedCommunicator, DistributedImpl, TorchDistributedImpl, destroy_distributed, register_plugin
from .info import DistributedInfo, get_tp_info, reset_tp_info, set_tp_info, try_get_tp_info

__all__ = [
    "DistributedInfo", "get_tp_info", "set_tp_info", "try_get_tp_info", "reset_tp_info",
    "DistributedCommunicator", "DistributedImpl", "TorchDistributedImpl", "destroy_distributed",
    "register_plugin",
]
