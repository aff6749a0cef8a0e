from .server import tokenize_worker

__all__ = ["tokenize_worker"]
