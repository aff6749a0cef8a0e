"""``python -m minisgl.shell --model ...``: interactive chat in the terminal."""

from minisgl.server import launch_server

if __name__ == "__main__":
    launch_server(run_shell=True)
