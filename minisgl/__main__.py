from minisgl.server import launch_server


def main() -> None:
    """Console entry point (``minisgl`` after ``pip install``): same as
    ``python -m minisgl``."""
    launch_server()


if __name__ == "__main__":
    main()
