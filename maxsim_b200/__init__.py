"""maxsim_b200 -- B200-native (sm_100a) compressed late-interaction scoring.

Drop-in for the reference ``maxsim`` package's GPU path: the same public names
(``Index``/``Corpus``, ``Reranker``, ``SearchResult``, ``pack_signs``,
``to_device``, ``score``, ``maxsim``, ``topk_maxsim``, the residual cascade
API) over ``libmaxsim_b200.so``.  ``maxsim_b200._maxsim_cuda`` reproduces the
reference's native extension module and can be installed as
``maxsim._maxsim_cuda``.

Importing the package loads the CUDA library; it fails loudly when the library
has not been built -- there is no CPU fallback.
"""

from maxsim_b200._api import PackedDocs, maxsim, pack_signs, score, to_device, topk_maxsim
from maxsim_b200.cascade import (
    BinaryResidualPackedDocs,
    ResidualInt4PackedDocs,
    binary_cascade_topk,
    binary_prefix_score,
    binary_residual_score,
    binary_residual_to_device,
    pack_binary_residual_int4,
    cascade_topk,
    pack_residual_int4,
    prefix_score,
    prefix_topk,
    residual_int4_to_device,
    residual_score,
)
from maxsim_b200.experimental import (
    DimCentroidCalibration,
    Int4PackedDocs,
    dim_centroid_maxsim,
    fit_dim_centroid_calibration,
    pack_dim_centroid_signs,
    topk_dim_centroid_maxsim,
    transform_query_dim_centroids,
    int4_maxsim,
    int4_maxsim_int8q,
    int4_to_device,
    pack_int4_symmetric,
    topk_int4_maxsim,
)
from maxsim_b200.sdk import MODE_PRESETS, Corpus, CorpusMemoryReport, Index, Reranker, SearchResult
from maxsim_b200.loader import load_reranker, load_resident_corpus

__all__ = [
    "PackedDocs",
    "Corpus",
    "Index",
    "load_reranker",
    "load_resident_corpus",
    "Reranker",
    "SearchResult",
    "CorpusMemoryReport",
    "MODE_PRESETS",
    "ResidualInt4PackedDocs",
    "Int4PackedDocs",
    "pack_signs",
    "to_device",
    "score",
    "maxsim",
    "topk_maxsim",
    "pack_int4_symmetric",
    "int4_to_device",
    "int4_maxsim",
    "int4_maxsim_int8q",
    "topk_int4_maxsim",
    "pack_residual_int4",
    "residual_int4_to_device",
    "prefix_score",
    "prefix_topk",
    "residual_score",
    "cascade_topk",
    "DimCentroidCalibration",
    "fit_dim_centroid_calibration",
    "pack_dim_centroid_signs",
    "transform_query_dim_centroids",
    "dim_centroid_maxsim",
    "topk_dim_centroid_maxsim",
    "BinaryResidualPackedDocs",
    "pack_binary_residual_int4",
    "binary_residual_to_device",
    "binary_prefix_score",
    "binary_residual_score",
    "binary_cascade_topk",
]
