"""StepPipeline (host buffers, graphed layer-steps, copies on side streams)
returns exactly what the eager public API returns for the same inputs, over
several steps with changing queries and sequence lengths and both buffers of
the double-buffering in use."""
import math

import numpy as np
import pytest
import torch

from amass_kv_b200 import attention as A
from amass_kv_b200 import selection as S
from amass_kv_b200.pipeline import StepPipeline
from amass_kv_b200.workloads import make_quad_case_gpu

pytestmark = pytest.mark.gpu


def test_pipeline_matches_eager():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(4)
    ctxs = rng.integers(2000, 9000, 6)
    L, n_kv, G, d = 2, 8, 4, 128
    b = make_quad_case_gpu(dev, seed=11, ctxs=ctxs, n_kv=n_kv, G=G, d=d,
                           page=16, r=2, v_bits=4, layers=L)
    R, MP = len(ctxs), b["MP"]
    st = S.QuadState(dev, num_layers=1, num_blocks=1, n_kv=n_kv, G=G,
                     head_dim=d, page=16, max_reqs=R, max_pages=MP, rank=2,
                     budget=0.05, v_bits=4, combine="nrm")
    st.quad_mu, st.mu_scale = b["quad_mu"], b["mu_scale"]
    st.quad_V, st.V_scale, st.quad_sig2 = b["quad_V"], b["V_scale"], b["quad_sig2"]
    A.ensure_stage_b_buffers(st, dev, 128)
    scale = 1 / math.sqrt(d)
    pipe = StepPipeline(st, [b["kv_cache"][l] for l in range(L)],
                        b["block_table"], n_req=R, scale=scale,
                        q_shape=tuple(b["q"].shape[1:]), device=dev)
    steps = 5
    qs = [torch.randn(b["q"].shape[1:]).to(torch.bfloat16).pin_memory()
          for _ in range(steps)]
    sls = [(b["seq_lens"].cpu() - 3 * (steps - i)).pin_memory()
           for i in range(steps)]
    outs = [torch.zeros_like(qs[0]).pin_memory() for _ in range(steps)]
    for i in range(steps):
        pipe.submit(i % L, qs[i], sls[i], outs[i])
    pipe.synchronize()
    for i in range(steps):
        q = qs[i].to(dev)
        sl = sls[i].to(dev)
        ref = torch.zeros_like(q)
        S.select_pages_quad(st, i % L, q, b["block_table"], sl, R, scale)
        A.sparse_paged_decode_batched_cuda(q, b["kv_cache"][i % L],
                                           b["block_table"], sl, st, ref,
                                           scale=scale)
        torch.cuda.synchronize()
        assert torch.equal(outs[i], ref.cpu()), i
