"""GPU parity of the r8 low-rank scorer (reference selection/score.py:30-148)
against the golden vectors from the reference's Triton kernel and against
the oracle (log-sum-exp and token-max forms)."""
import numpy as np
import pytest
import torch

from amass_kv_b200 import selection as S
from amass_kv_b200.workloads import make_r8_case
from oracle import amass_oracle as O
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _state(dev, *, q, block_table, seq_lens, mu, mu_s, Vk, Vk_s, c, c_s, G,
           r, vk_bits, c_bits, page, MP, budget):
    NB, n_kv, d = mu.shape
    n_req = block_table.shape[0]
    st = S.R8State(dev, num_layers=1, num_blocks=NB, n_kv=n_kv, G=G,
                   head_dim=d, page=page, max_reqs=n_req, max_pages=MP,
                   rank=r, budget=budget, vk_bits=vk_bits, c_bits=c_bits)
    for dst, src in ((st.r8_mu, mu), (st.mu_scale, mu_s), (st.r8_Vk, Vk),
                     (st.Vk_scale, Vk_s), (st.r8_c, c), (st.c_scale, c_s)):
        dst[0].copy_(torch.from_numpy(np.ascontiguousarray(src)))
    st.score.fill_(float("nan"))
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    qd = q if isinstance(q, torch.Tensor) else t(q)
    return st, qd, t(block_table), t(seq_lens)


@pytest.mark.parametrize("name", ["r8_i8", "r8_i4"])
def test_r8_golden(name, dev):
    z = load_golden(name)
    G, r, vkb, cb, page, MP, n_kv, d = [int(x) for x in z["meta"]]
    q = torch.from_numpy(z["q"]).view(torch.bfloat16).to(dev)
    st, q, bt, sl = _state(dev, q=q, block_table=z["block_table"],
                           seq_lens=z["seq_lens"], mu=z["mu"], mu_s=z["mu_s"],
                           Vk=z["Vk"], Vk_s=z["Vk_s"], c=z["c"], c_s=z["c_s"],
                           G=G, r=r, vk_bits=vkb, c_bits=cb, page=page, MP=MP,
                           budget=float(z["budget"][0]))
    n_req = bt.shape[0]
    S.select_pages_r8(st, 0, q, bt, sl, n_req, float(z["scale"][0]))
    torch.cuda.synchronize()
    sc = st.score.cpu().numpy()
    for rq, n in enumerate(z["n_sel_hi"]):
        np.testing.assert_allclose(sc[rq, :, :n], z["score"][rq, :, :n],
                                   rtol=1e-4, atol=1e-4)
    ref = np.where(np.isnan(z["score"]), -np.inf, z["score"])
    assert O.selection_diff_ok(st.page_table.cpu().numpy(),
                               st.page_cnt.cpu().numpy(), z["page_table"],
                               z["page_cnt"], ref)


@pytest.mark.parametrize("seed,vkb,cb,agg", [(41, 8, 8, "lse"),
                                             (42, 4, 4, "lse"),
                                             (43, 8, 4, "tokmax")])
def test_r8_random_vs_oracle(seed, vkb, cb, agg, dev):
    rng = np.random.default_rng(seed)
    ctxs = tuple(int(x) for x in rng.integers(300, 5000, size=5))
    c = make_r8_case(seed, n_req=5, n_kv=8, G=4, d=128, ctxs=ctxs, r=8,
                     vk_bits=vkb, c_bits=cb)
    st, q, bt, sl = _state(dev, q=c.q.astype(np.float32), block_table=c.block_table,
                           seq_lens=c.seq_lens, mu=c.mu, mu_s=c.mu_s, Vk=c.Vk,
                           Vk_s=c.Vk_s, c=c.c, c_s=c.c_s, G=4, r=8,
                           vk_bits=vkb, c_bits=cb, page=16, MP=c.MP,
                           budget=0.05)
    q = q.to(torch.bfloat16)
    S.select_pages_r8(st, 0, q, bt, sl, 5, c.scale, token_agg=agg)
    torch.cuda.synchronize()
    npg, nsh, b = O.derive_page_params(c.seq_lens, 0.05, 16, 1, 1)
    ref = O.r8_score(c.q, c.mu, c.mu_s, c.Vk, c.Vk_s, c.c, c.c_s,
                     c.block_table, c.seq_lens, nsh, scale=c.scale, page=16,
                     G=4, r=8, vk_bits=vkb, c_bits=cb, MP=c.MP,
                     combine=agg)
    sc = st.score.cpu().numpy()
    for rq, n in enumerate(nsh):
        np.testing.assert_allclose(sc[rq, :, :n], ref[rq, :, :n], rtol=1e-4,
                                   atol=1e-4)
    refm = np.where(np.isnan(ref), -np.inf, ref)
    tab, cnt = O.topb_select(refm, npg, nsh, b, sink=1, MP=c.MP)
    assert O.selection_diff_ok(st.page_table.cpu().numpy(),
                               st.page_cnt.cpu().numpy(), tab, cnt, refm)
