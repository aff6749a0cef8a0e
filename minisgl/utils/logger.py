"""Per-process coloured logger with rank-0 helpers.

Format: ``[date|time|pid=..|core|rank=r] LEVEL message`` (the pid part when
LOG_PID is set, the rank part once the TP rank is known). LOG_LEVEL selects
the level.
"""

from __future__ import annotations

import logging
import os
import sys

_LEVELS = {"DEBUG": logging.DEBUG, "INFO": logging.INFO, "WARNING": logging.WARNING,
           "ERROR": logging.ERROR, "CRITICAL": logging.CRITICAL}
_COLORS = {"DEBUG": "\033[36m", "INFO": "\033[32m", "WARNING": "\033[33m", "ERROR": "\033[31m",
           "CRITICAL": "\033[35m"}
_RESET, _BOLD = "\033[0m", "\033[1m"


class _Formatter(logging.Formatter):
    def __init__(self, tag: str, use_rank: bool | None) -> None:
        super().__init__()
        self.tag = tag
        self.use_rank = use_rank

    def format(self, record: logging.LogRecord) -> str:
        from minisgl.parallel.info import get_cp_info, get_dp_info, try_get_tp_info

        tag = self.tag
        info = get_cp_info() or get_dp_info() or try_get_tp_info()
        if info is not None and self.use_rank is not False:
            tag = f"{tag}|core|rank={info.rank}"
        stamp = self.formatTime(record, "%Y-%m-%d|%H:%M:%S")
        color = _COLORS.get(record.levelname, "")
        return f"{_BOLD}[{stamp}{tag}]{_RESET} {color}{record.levelname:<8}{_RESET} {record.getMessage()}"


class MiniLogger(logging.Logger):
    """Logger with *_rank0 variants that only emit on the primary TP rank."""

    def _rank0(self) -> bool:
        from minisgl.parallel.info import get_cp_info, get_dp_info, try_get_tp_info

        info = get_cp_info() or get_dp_info() or try_get_tp_info()
        return info is None or info.is_primary()

    def info_rank0(self, msg, *args, **kwargs):
        if self._rank0():
            self.info(msg, *args, **kwargs)

    def debug_rank0(self, msg, *args, **kwargs):
        if self._rank0():
            self.debug(msg, *args, **kwargs)

    def warning_rank0(self, msg, *args, **kwargs):
        if self._rank0():
            self.warning(msg, *args, **kwargs)

    def critical_rank0(self, msg, *args, **kwargs):
        if self._rank0():
            self.critical(msg, *args, **kwargs)


def init_logger(name: str, suffix: str = "", *, level: str | None = None, use_pid: bool | None = None,
                use_tp_rank: bool | None = None) -> MiniLogger:
    old_cls = logging.getLoggerClass()
    logging.setLoggerClass(MiniLogger)
    try:
        logger = logging.getLogger(name)
    finally:
        logging.setLoggerClass(old_cls)
    if not isinstance(logger, MiniLogger):  # created earlier with another class
        logger.__class__ = MiniLogger
    lvl = (level or os.getenv("LOG_LEVEL", "INFO")).upper()
    logger.setLevel(_LEVELS.get(lvl, logging.INFO))
    if use_pid is None:
        use_pid = os.getenv("LOG_PID", "0").lower() in ("1", "true", "yes")
    tag = ""
    if use_pid:
        tag += f"|pid={os.getpid()}"
    if suffix:
        tag += f"|{os.path.basename(suffix)}"
    logger.handlers.clear()
    handler = logging.StreamHandler(sys.stdout)
    handler.setFormatter(_Formatter(tag, use_tp_rank))
    logger.addHandler(handler)
    logger.propagate = False
    return logger  # type: ignore[return-value]
