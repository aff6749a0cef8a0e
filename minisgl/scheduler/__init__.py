from .config import SchedulerConfig
from .scheduler import Scheduler

__all__ = ["Scheduler", "SchedulerConfig"]
