"""B200-native engine for the BSSCL-GBM binary-logloss hot path.

``HybridHistGBMNumbaV1_0_1`` keeps the reference estimator's API
(src/bsscl_gbm/__init__.py:5-9 exports the same class name); every boosting
round and every predict runs in libgbm_b200.so on an NVIDIA B200.
"""

from .estimator import HybridHistGBMNumbaV1_0_1, HybridHistGBMRegressorV1_0_1
from ._lib import Engine, Sampler, GbmParams, build, lib

__all__ = ["HybridHistGBMNumbaV1_0_1", "HybridHistGBMRegressorV1_0_1", "Engine", "Sampler", "GbmParams", "build", "lib"]
__version__ = "0.1.0"
