# minisgl on B200: CUDA 12.9 toolchain (nvcc cross-compiles sm_100a), the
# engine built and installed as a package, the server as the entry point.
#
#   docker build -t minisgl .
#   docker run --gpus all --ipc=host -p 1919:1919 -v /models:/models minisgl \
#       --model /models/Qwen3-32B --tp 8 --host 0.0.0.0
ARG CUDA_IMAGE=nvidia/cuda:12.9.1-devel-ubuntu24.04
FROM ${CUDA_IMAGE}

ENV DEBIAN_FRONTEND=noninteractive \
    PYTHONUNBUFFERED=1 \
    PIP_NO_CACHE_DIR=1 \
    TORCH_CUDA_ARCH_LIST=10.0a
RUN apt-get update && apt-get install -y --no-install-recommends \
        python3 python3-dev python3-venv git ninja-build && \
    rm -rf /var/lib/apt/lists/*

RUN python3 -m venv /opt/venv
ENV PATH=/opt/venv/bin:$PATH
# torch with CUDA 12.8+ kernels (its bundled NCCL serves the NCCL baseline path)
RUN pip install "torch>=2.6" --index-url https://download.pytorch.org/whl/cu128 && \
    pip install setuptools wheel ninja

WORKDIR /src
COPY pyproject.toml setup.py README.md ./
COPY minisgl ./minisgl
# the extension is compiled for sm_100a only (see setup.py); the build needs
# no GPU
RUN pip install --no-build-isolation ".[bench]" && python -c "import minisgl._C"

RUN useradd --create-home --uid 1001 minisgl
USER minisgl
ENV HF_HOME=/home/minisgl/.cache/huggingface
EXPOSE 1919
ENTRYPOINT ["python", "-m", "minisgl"]
CMD ["--help"]
