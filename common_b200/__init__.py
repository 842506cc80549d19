"""common_b200 -- B200-native (sm_100a) backend for the almostrealism/common Qwen3 forward step.

The compute lives in libqwen3_b200.so (common_b200/csrc, C ABI in include/qwen3_b200.h);
this package holds its build script, its ctypes binding and a host-side mirror of the
reference's Qwen3 runtime API.
"""
from . import native  # noqa: F401
from .qwen3 import (AutoregressiveModel, CompiledModel, Qwen3, Qwen3Config, StateDictionary,  # noqa: F401
                    infer_config, synthetic_state_dict)

__all__ = ["native", "Qwen3", "Qwen3Config", "StateDictionary", "CompiledModel", "AutoregressiveModel",
           "infer_config", "synthetic_state_dict"]
