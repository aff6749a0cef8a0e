from .launch import launch_server

__all__ = ["launch_server"]
