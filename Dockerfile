# B200 (sm_100a) runtime image: CUDA 12.9 toolkit for the in-tree extension build, PyTorch with sm_100 support.
FROM nvidia/cuda:12.9.1-devel-ubuntu24.04
RUN apt-get update && apt-get install -y --no-install-recommends python3 python3-pip python3-venv git \
    && rm -rf /var/lib/apt/lists/*
RUN python3 -m venv /opt/venv
ENV PATH=/opt/venv/bin:$PATH
RUN pip install --no-cache-dir torch numpy pyyaml tokenizers sentencepiece fastapi uvicorn pydantic psutil \
    nvidia-ml-py transformers datasets
WORKDIR /opt/quantaweave
COPY . .
# compile every CUDA source for sm_100a into quantaweave_b200/_C (in tree)
RUN python setup.py build_ext --inplace
ENV PYTHONPATH=/opt/quantaweave
CMD ["python", "-m", "quantaweave_b200.tools.serve", "--help"]
