from .llm import LLM, RequestAllFinished

__all__ = ["LLM", "RequestAllFinished"]
