"""minisgl: a Blackwell-native (sm_100a) LLM inference engine with the public
surface of mini-sglang (OpenAI-compatible server, shell, offline LLM API)."""

__version__ = "0.1.0"
