"""B200-native Voxtral decode path: backbone decode loop + flow-matching transformer.

The compute lives in libvoxtral_b200.so (hand-written CUDA for sm_100a behind the C ABI
of include/voxtral_b200.h); this package is the host-side mirror of the reference's
VoxtralEngine API.  The directory name is not a Python identifier, so import it with
importlib:

    vx = importlib.import_module("webgpu-voxtral_b200")
"""
from .engine import (TTSResult, VoxtralEngine, VoxtralError, default_config, header_symbols, library_path,
                     load_library, nccl_unique_id, tp_init)
from . import synth

__all__ = ["VoxtralEngine", "VoxtralError", "TTSResult", "default_config", "header_symbols", "library_path",
           "load_library", "nccl_unique_id", "tp_init", "synth"]
