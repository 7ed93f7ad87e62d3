"""`tiny_metal_nn` import name for users of the reference's Python module
(src/python/tmnn_pybind.cpp: `tiny_metal_nn.Trainer.from_config`, the typed
errors).  Everything is the B200 package `tmnn_b200`."""
from tmnn_b200 import (ClosedError, ConcurrentTrainingStepError,  # noqa: F401
                       ConfigError, DTypeError, FullyFusedMLP, NerfField,
                       Trainer, TmnnError, dp_unique_id)

__version__ = "0.1.0a2+b200"
__all__ = ["Trainer", "ClosedError", "ConcurrentTrainingStepError",
           "ConfigError", "DTypeError", "TmnnError", "FullyFusedMLP",
           "NerfField", "dp_unique_id"]
