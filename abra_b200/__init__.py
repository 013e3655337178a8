"""abra_b200 -- B200-native (sm_100a) Q4_K x Q8_1 decode path (with its Q6_K leg).

The compute lives in libabra_b200.so (hand-written CUDA for sm_100a behind a
C ABI, include/abra_b200.h).  This package binds it with ctypes and mirrors
the reference's operator interface (abra_b200.q4k).  Importing it without the
built library raises; there is no CPU fallback.
"""
from . import _lib
from ._lib import AbraError
from .q4k import (
    ARCH_SM100,
    CANDIDATE_AUTOTUNED_DISPATCH,
    QK8_1,
    QK_K,
    Q4K_BYTES,
    Q81_BYTES,
    Q4KCandidateSpec,
    device_error,
    gen_q4k,
    gen_uniform_f32,
    get_all_candidate_ids,
    get_autotuned_candidate_for_shape,
    get_candidate_name,
    get_candidate_spec,
    launch_custom_reference_q8_1_quantizer,
    launch_q4k_autotuned,
    launch_q4k_autotuned_combined_pipeline,
    launch_q4k_candidate,
    launch_q4k_candidate_combined_pipeline,
    launch_quantize_f32_to_q8_1,
    load_tuning_table,
    mmvq,
    mmvq_kshard,
    mmvq_packed,
    mmvq_partials,
    mmvq_rmsnorm,
    mmvq_swiglu,
    mmvq_tc,
    plan_info,
    q4k_nbytes,
    pack_q4k,
    q8_1_nbytes,
    register_autotuned_table_entry,
    rmsnorm_quantize_q8_1,
    slice_start,
)
from .q6k import (
    Q6K_BYTES,
    Q6KCandidateSpec,
    gen_q6k,
    mmvq_q6k,
    mmvq_q6k_kshard,
    mmvq_q6k_partials,
    q6k_candidates,
    q6k_nbytes,
    q6k_tune_get,
    q6k_tune_set,
)

__version__ = _lib.lib.abra_version().decode()
LIB_PATH = _lib.LIB_PATH
