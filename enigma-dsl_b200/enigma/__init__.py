"""Enigma on B200: the Enigma DSL surface with sm_100a CUDA kernels behind it."""
from . import cuda_ops as cuda_ops
