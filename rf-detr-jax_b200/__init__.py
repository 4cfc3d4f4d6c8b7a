"""B200-native (sm_100a) backend for RF-DETR-JAX's training hot path.

The package directory is ``rf-detr-jax_b200``; it is imported as ``rfdetr_jax_b200``
(``__graft_entry__.load_package()`` registers it under that name).

Components (each a thin host wrapper over ``librfdetr_b200.so``, see ``include/rfdetr_b200.h``):

* :mod:`.ops`     -- multi-scale deformable attention, sampler ``"cuda"``, forward + backward, and
  its query -> (locations, weights) prologue;
* :mod:`.topk`    -- two-stage query selection (class max + top-k) and ``select_rows``;
* :mod:`.matcher` -- matching cost and exact batched assignment (SciPy-identical);
* :mod:`.postprocess` -- inference post-process (top-k over all query/class pairs);
* :mod:`.losses` -- IA-BCE or focal and matched-pair box losses of stacked layers, with gradients;
* :mod:`.collective` -- the data-parallel gradient all-reduce over NVLink peer memory.
"""

from . import _native
from ._native import check_device_status, set_tuning
from .collective import PeerAllReduce
from .matcher import CriterionConfig, build_cost_matrix, hungarian_match, match_stacked
from .ops import (MSDeformAttnFunction, MSDeformAttnPrologueFunction, ms_deform_attn, ms_deform_attn_core,
                  ms_deform_attn_core_rows, msda_prologue)
from .losses import SetLossFunction, set_losses
from .postprocess import post_process
from .topk import select_rows, top_k, two_stage_topk

__all__ = [
    "CriterionConfig",
    "MSDeformAttnFunction",
    "PeerAllReduce",
    "build_cost_matrix",
    "check_device_status",
    "hungarian_match",
    "match_stacked",
    "ms_deform_attn",
    "ms_deform_attn_core",
    "ms_deform_attn_core_rows",
    "msda_prologue",
    "MSDeformAttnPrologueFunction",
    "post_process",
    "set_losses",
    "set_tuning",
    "SetLossFunction",
    "select_rows",
    "top_k",
    "two_stage_topk",
]

LIB_PATH = _native.LIB_PATH
