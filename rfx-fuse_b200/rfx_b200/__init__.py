"""rfx_b200: B200-native forest growth and proximity behind the RFXFuse Python API.

    import rfx_b200 as RFXFuse
    rf = RFXFuse.RandomForestClassifier(nsample=n, ntree=100, mtry=4, minndsize=1,
                                        compute_proximity=True)
    rf.fit(X, y)
    rf.get_oob_error(); rf.feature_importances_(); rf.get_proximity_matrix()

All computation runs in librfx_b200.so (hand-written sm_100a CUDA); see include/rfx_b200.h.
"""
from ._abi import Context, RfxError, cached_bytes, empty_cache, load_library  # noqa: F401
from .model_io import LoadedModel, load  # noqa: F401
from .impute import rfx_impute_proximity, rfx_impute_topk_mean, rfx_impute_topk_median  # noqa: F401
from .forest import (TaskType, RandomForestClassifier, RandomForestRegressor,  # noqa: F401
                     RandomForestUnsupervised, calculate_maxnode, detect_categorical)

__all__ = ["TaskType", "RandomForestClassifier", "RandomForestRegressor", "RandomForestUnsupervised",
           "Context", "RfxError", "load_library", "cached_bytes", "empty_cache",
           "calculate_maxnode", "detect_categorical",
           "LoadedModel", "load", "rfx_impute_proximity", "rfx_impute_topk_mean",
           "rfx_impute_topk_median"]
