"""B200-native in-HBM search path of GustANN.

Public surface:
  GustANN, GustANNConfig, GustANNStats, GustANNError   host API (api.py)
  UINT8, FLOAT                                         data types
  formats                                              on-disk index formats
  index                                                synthetic data + index builder

Importing the package does not load the CUDA library; ``gustann_b200.api``
does, and raises if it is not built.
"""
from .formats import FLOAT, UINT8  # noqa: F401

__all__ = ["GustANN", "GustANNConfig", "GustANNStats", "GustANNError", "UINT8", "FLOAT"]


def __getattr__(name):
    if name in ("GustANN", "GustANNConfig", "GustANNStats", "GustANNError", "pivot_sample"):
        from . import api
        return getattr(api, name)
    raise AttributeError(name)
