"""amass_kv_b200 -- the AMASS decode-time sparse paged-attention hot path on
B200 (sm_100a).

Host layer (this package, Python/PyTorch) over ``libamass_b200.so`` (CUDA C++,
C ABI in ``include/amass_b200.h``):

  selection  QuadState, derive_page_params, quad_score_cuda, topb_select_cuda,
             select_pages, select_pages_quad                      (Stage A)
  attention  ResidentVSource, ensure_stage_b_buffers,
             sparse_paged_decode_batched_cuda                     (Stage B)

The configuration object stays the reference's own ``AmassConfig``; callers
pass its fields (budget, coverage, combine, ...) to the state constructors.
"""
