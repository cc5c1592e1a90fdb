"""oasis_b200: B200-native (sm_100a) Oasis-500M per-frame generation.

The directory is named open-oasis_b200; it is imported as the package
`oasis_b200` (see __graft_entry__.load_package). Compute lives entirely in
liboasis_b200.so (hand-written CUDA for sm_100a, C ABI in include/oasis_b200.h);
Python here is host plumbing: weight packing, conditioning, buffers, graphs.

Modules
  host            constants, conditioning, schedule, RoPE tables (CPU fp32)
  weights         seeded random-init weights and their device packing
  engine          native API: dit_forward, ddim_step, vae_decode, FrameEngine
  oasis_inference drop-in functions with the reference's names and call shapes
  parallel        session data parallelism across GPUs
  build           nvcc build of the shared library
"""
from . import host  # noqa: F401
from ._lib import OasisError, OasisLibraryError, load as load_library  # noqa: F401

__version__ = "0.1.0"


def __getattr__(name):
    # engine/weights import torch CUDA plumbing lazily so CPU-only imports stay light
    if name in ("engine", "weights", "oasis_inference", "parallel"):
        import importlib

        return importlib.import_module(f"{__name__}.{name}")
    raise AttributeError(name)
