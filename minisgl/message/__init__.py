from .backend import AbortBackendMsg, BaseBackendMsg, BatchBackendMsg, ExitMsg, UserMsg
from .frontend import BaseFrontendMsg, BatchFrontendMsg, UserReply
from .tokenizer import AbortMsg, BaseTokenizerMsg, BatchTokenizerMsg, DetokenizeMsg, TokenizeMsg

__all__ = [
    "AbortMsg", "AbortBackendMsg", "BaseBackendMsg", "BatchBackendMsg", "ExitMsg", "UserMsg",
    "BaseTokenizerMsg", "BatchTokenizerMsg", "DetokenizeMsg", "TokenizeMsg", "BaseFrontendMsg",
    "BatchFrontendMsg", "UserReply",
]
