"""GPU parity of the page summary build (quad, CLSE, r8 slabs) against the
reference's quad_build_tail goldens and the oracle restatement.

Eigenvectors are unique up to sign, so V columns and coordinates are
compared up to a per-column sign; mu codes within one code, scales and
eigenvalues within 0.5%, tags bit-exact (same checks as the oracle pin)."""
import numpy as np
import pytest
import torch

from amass_kv_b200 import summaries as SU
from amass_kv_b200.selection import QuadState, R8State
from oracle import amass_oracle as O
from tests.conftest import bits_to_f32, load_golden
from tests.test_oracle_golden import _tail_pages, check_summary

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _slabs(st, l, lse):
    f = lambda t: t[l].cpu().numpy()                       # noqa: E731
    got = dict(mu=f(st.quad_mu), mu_s=f(st.mu_scale), sig2=f(st.quad_sig2),
               V=f(st.quad_V), V_s=f(st.V_scale),
               tag=st.quad_tag[l].view(torch.int16).cpu().numpy())
    if lse:
        got.update(c=f(st.quad_c), c_s=f(st.c_scale), resid=f(st.quad_resid))
    return got


@pytest.mark.parametrize("name", ["build_quad_i4", "build_clse_i8"])
def test_build_tail_matches_reference(name, dev):
    z = load_golden(name)
    (L, NB, n_kv, d, r, vb, cb, ctok, lse), blocks = _tail_pages(z)
    n_req = z["block_table"].shape[0]
    st = QuadState(dev, num_layers=L, num_blocks=NB, n_kv=n_kv, G=4,
                   head_dim=d, page=16, max_reqs=n_req,
                   max_pages=z["block_table"].shape[1], rank=r, budget=0.1,
                   v_bits=vb, coords="lse" if lse else "none", c_bits=cb,
                   c_grain="token" if ctok else "page")
    K = torch.from_numpy(z["K"]).view(torch.bfloat16).to(dev)  # (L,NB,t,kv,d)
    bt = torch.from_numpy(z["block_table"]).to(dev)
    sl = torch.from_numpy(z["seq_lens"]).to(dev)
    n = SU.quad_build_tail(st, [K[l] for l in range(L)], bt, sl, n_req)
    torch.cuda.synchronize()
    assert n == L * n_req
    for l in range(L):
        check_summary(z, _slabs(st, l, lse), l, blocks)


@pytest.mark.parametrize("d,r,v_bits,coords,c_bits,c_grain", [
    (128, 2, 4, "none", 4, "token"),
    (128, 4, 8, "lse", 4, "token"),
    (64, 8, 8, "lse", 8, "page"),
])
def test_bulk_build_vs_oracle(d, r, v_bits, coords, c_bits, c_grain, dev):
    rng = np.random.default_rng(d + r)
    NB, n_kv, L = 40, 4, 2
    K = rng.standard_normal((L, NB, 16, n_kv, d)).astype(np.float32)
    K[..., :5] *= 3.0
    Kb = torch.from_numpy(K).to(torch.bfloat16)
    K = Kb.float().numpy()
    ctxs = [300, 160, 33]
    bt = np.zeros((3, 32), np.int32)
    perm = rng.permutation(NB)
    o = 0
    for i, c in enumerate(ctxs):
        n = -(-c // 16)
        bt[i, :n] = perm[o:o + n]
        o += n
    st = QuadState(dev, num_layers=L, num_blocks=NB, n_kv=n_kv, G=4,
                   head_dim=d, page=16, max_reqs=3, max_pages=32, rank=r,
                   budget=0.1, v_bits=v_bits, coords=coords, c_bits=c_bits,
                   c_grain=c_grain)
    Kd = Kb.to(dev)
    SU.quad_build_bulk(st, [Kd[l] for l in range(L)],
                       torch.from_numpy(bt).to(dev),
                       torch.tensor(ctxs, dtype=torch.int32, device=dev), 3,
                       max_fin=32)
    torch.cuda.synchronize()
    fin = [c // 16 for c in ctxs]
    blocks = sorted({int(bt[i, p]) for i in range(3) for p in range(fin[i])})
    meta = np.array([L, NB, n_kv, d, r, v_bits, c_bits,
                     1 if c_grain == "token" else 0,
                     1 if coords == "lse" else 0], np.int64)
    for l in range(L):
        s = O.page_summary(K[l][blocks], r, v_bits=v_bits, coords=coords,
                           c_bits=c_bits, c_grain=c_grain)
        z = {"meta": meta, "seq_lens": np.array(ctxs), "block_table": bt,
             "mu": np.zeros((L, NB, n_kv, d), np.int8)}
        zz = dict(z)
        for key, src in (("mu", "mu_code"), ("mu_s", "mu_s"), ("sig2", "sig2"),
                         ("V", "V_code"), ("V_s", "V_s"), ("c", "c_code"),
                         ("c_s", "c_s"), ("resid", "resid")):
            if src in s:
                arr = np.zeros((L, NB) + s[src].shape[1:], s[src].dtype)
                arr[l, blocks] = s[src]
                zz[key] = arr
        tag = np.zeros((L, NB, n_kv, 8), np.int16)
        tag[l, blocks] = (s["tag"].view(np.uint32) >> 16).astype(
            np.uint16).view(np.int16)
        zz["tag"] = tag
        check_summary(zz, _slabs(st, l, coords == "lse"), l, blocks)


def test_r8_state_build_matches_oracle(dev):
    rng = np.random.default_rng(5)
    NB, n_kv, d = 24, 2, 128
    K = torch.from_numpy(rng.standard_normal((NB, 16, n_kv, d)).astype(
        np.float32)).to(torch.bfloat16)
    st = R8State(dev, num_layers=1, num_blocks=NB, n_kv=n_kv, G=4,
                 head_dim=d, page=16, max_reqs=1, max_pages=8, rank=8,
                 budget=0.1, vk_bits=8, c_bits=8)
    blocks = torch.arange(NB, dtype=torch.int32, device=dev)
    SU.summarize_pages(st, [K.to(dev)], blocks)
    torch.cuda.synchronize()
    s = O.page_summary(K.float().numpy(), 8, v_bits=8, coords="lse",
                       c_bits=8, c_grain="token")
    np.testing.assert_allclose(st.mu_scale[0].cpu().float().numpy(),
                               s["mu_s"].astype(np.float32), rtol=2e-3)
    # coordinates up to a per-column sign, per-token scales
    cg = st.r8_c[0].cpu().numpy().astype(np.float32) * \
        st.c_scale[0].cpu().float().numpy()[..., None]
    cr = s["c_code"].astype(np.float32) * s["c_s"].astype(np.float32)[..., None]
    sg = np.sign((cg * cr).sum(axis=2, keepdims=True))
    assert np.abs(cr - sg * cg).max() <= 1.5 * s["c_s"].astype(np.float32).max()


def test_tag_stale_matches_reference(dev):
    """The staleness kernel marks exactly the blocks the reference's tag
    pass selects, in order (tag-channel edits and a NaN tag; edits outside
    the tag channels or the page-final token stay fresh)."""
    import ctypes
    from amass_kv_b200 import _lib
    z = load_golden("build_delta_tags")
    K = torch.from_numpy(z["K"]).view(torch.bfloat16).to(dev)
    tag = torch.from_numpy(z["tag"]).view(torch.bfloat16).to(dev)
    L = K.shape[0]
    bt = torch.from_numpy(z["block_table"]).to(dev)
    sl = torch.from_numpy(z["seq_lens"]).to(dev)
    mf = int(z["max_fin"][0])
    cand = SU.delta_blocks(bt, sl, bt.shape[0], 16, mf)
    out = torch.empty_like(cand)
    cnt = torch.zeros(1, dtype=torch.int32, device=dev)
    ks = [K[l] for l in range(L)]
    arr = (ctypes.c_void_p * L)(*[k.data_ptr() for k in ks])
    _lib.call("amass_tag_stale", ctypes.cast(arr, ctypes.c_void_p), L,
              ks[0].stride(0), ks[0].stride(1), ks[0].stride(2),
              tag.data_ptr(), 0, K.shape[1], K.shape[3], tag.shape[-1], 16,
              cand.data_ptr(), cand.numel(), out.data_ptr(), cnt.data_ptr(),
              _lib.stream_of(dev))
    o = out.cpu().numpy()
    assert o[o >= 0].tolist() == z["stale"].tolist()
    assert int(cnt.item()) == len(z["stale"])


def test_delta_rebuild_equals_bulk(dev):
    """First delta (NaN tags) rebuilds every finalized block; a second finds
    nothing; after keys of two blocks change, the delta result equals a
    bulk rebuild of the changed keys, slab for slab."""
    rng = np.random.default_rng(9)
    L, n_kv, d, page = 3, 4, 128, 16
    ctxs = [300, 517, 64, 129]
    npg = [(c + page - 1) // page for c in ctxs]
    NB = sum(npg) + 5
    perm = rng.permutation(NB).astype(np.int32)
    MP = max(npg)
    bt_np = np.zeros((len(ctxs), MP), np.int32)
    o = 0
    for i, n in enumerate(npg):
        bt_np[i, :n] = perm[o:o + n]
        o += n
    bt = torch.from_numpy(bt_np).to(dev)
    sl = torch.tensor(ctxs, dtype=torch.int32, device=dev)
    K = torch.randn((L, NB, page, n_kv, d), device=dev).to(torch.bfloat16)
    mk = lambda: QuadState(dev, num_layers=L, num_blocks=NB, n_kv=n_kv, G=4,  # noqa: E731
                           head_dim=d, page=page, max_reqs=len(ctxs),
                           max_pages=MP, rank=2, budget=0.1, v_bits=4)
    st, ref = mk(), mk()
    mf = max(c // page for c in ctxs)
    n_fin = sum(c // page for c in ctxs)
    ks = [K[l] for l in range(L)]
    assert SU.quad_build_delta(st, ks, bt, sl, len(ctxs), mf) == L * n_fin
    assert SU.quad_build_delta(st, ks, bt, sl, len(ctxs), mf) == 0
    K[2, int(bt_np[1, 7]), page - 1, 3, 0] += 2.0
    K[0, int(bt_np[0, 2]), page - 1, 0, 7] -= 1.0
    assert SU.quad_build_delta(st, ks, bt, sl, len(ctxs), mf) == 2 * L
    SU.quad_build_bulk(ref, ks, bt, sl, len(ctxs), mf)
    torch.cuda.synchronize()
    fin = [int(bt_np[r, p]) for r in range(len(ctxs))
           for p in range(ctxs[r] // page)]
    for name in ("quad_mu", "mu_scale", "quad_V", "V_scale", "quad_sig2",
                 "quad_tag"):
        a = getattr(st, name)[:, fin].view(torch.int8)
        b = getattr(ref, name)[:, fin].view(torch.int8)
        assert torch.equal(a, b), name
