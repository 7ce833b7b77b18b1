"""qwen3.c token mixers on B200: the CUDA backend (libcoli_cuda.so) and its
host-side binding. The compute lives in csrc/*.cu behind the C ABI of
include/backend_cuda.h; this package only builds and binds it."""
from . import coli_cuda, peer, sharding, snapshot, stack, synth  # noqa: F401
from .build import build, LIB  # noqa: F401
from .coli_cuda import Backend, BackendError, header_symbols, load_library  # noqa: F401
