"""B200-native (sm_100a) WnW decode hot path.

Public API:
  WnWConfig           -- head classes / chunk configuration (reference schema)
  B200WnWCache        -- drop-in for the reference WnWCache / WnWCppCache
  WnWSession          -- attention-patching session driving the cache hooks
  Planner             -- the native decode planner (reference pybind API)
  LlamaFamilyAdapter  -- adapter for HF Llama-family decoders

The CUDA kernels live in libwnw_b200.so (``python -m wnw_b200.build``); the
cache and kernel wrappers raise ImportError when it is missing.
"""
from wnw_b200.config import WnWConfig

__all__ = ["WnWConfig", "B200WnWCache", "WnWSession", "Planner", "LlamaFamilyAdapter"]


def __getattr__(name):
    if name == "B200WnWCache":
        from wnw_b200.cache import B200WnWCache
        return B200WnWCache
    if name == "WnWSession":
        from wnw_b200.session import WnWSession
        return WnWSession
    if name == "Planner":
        from wnw_b200.planner import Planner
        return Planner
    if name == "LlamaFamilyAdapter":
        from wnw_b200.adapters import LlamaFamilyAdapter
        return LlamaFamilyAdapter
    raise AttributeError(name)
