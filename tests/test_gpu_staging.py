"""GPU parity of the tier's staging lifecycle (write path): begin_step's five
ordered kernels (flushed-latch clear, collect + free, flush copy into the
pinned pool, staging-block allocation, slot mapping) and scatter_kv, through
the C ABI, against the reference's golden trace and the CPU oracle.

Bar: bit-exact -- vbo, flushed latches, the free stack and its top, the flush
list in order, v_slot_mapping, every pool / staging-pool byte, pool_valid and
the overflow latch.
"""
import numpy as np
import pytest
import torch

from amass_kv_b200 import tier as T
from oracle import amass_oracle as O
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _oracle_state(L, NB, n_kv, d, page, NV, MAXF, max_tokens):
    return dict(vbo=np.full(NB, -1, np.int32), vfl=np.zeros(NB, np.int32),
                stack=np.arange(NV, dtype=np.int32), top=NV,
                flist=np.zeros((MAXF, 2), np.int32), fcnt=0, ovf=0,
                vslot=np.full(max_tokens, -1, np.int64),
                v_pool=np.zeros((L, NV, page, n_kv, d), np.int16), MAXF=MAXF)


def _i16(t):
    return t.view(torch.int16).cpu().numpy()


def _check(stg, st, n_tok, pool, valid, o_pool, o_valid, tag):
    assert np.array_equal(stg.vbo.cpu().numpy(), st["vbo"]), tag
    assert np.array_equal(stg.v_flushed.cpu().numpy(), st["vfl"]), tag
    top = int(stg.v_free_top.item())
    assert top == st["top"], tag
    assert np.array_equal(stg.v_free_stack.cpu().numpy()[:top],
                          st["stack"][:top]), tag
    fc = int(stg.flush_cnt.item())
    assert fc == st["fcnt"], tag
    assert np.array_equal(stg.flush_list.cpu().numpy()[:fc],
                          st["flist"][:fc]), tag
    assert np.array_equal(stg.v_slot_mapping[:n_tok].cpu().numpy(),
                          st["vslot"][:n_tok]), tag
    assert int(stg.overflow.item()) == st["ovf"], tag
    assert np.array_equal(_i16(stg.v_pool), st["v_pool"]), tag
    assert np.array_equal(pool, o_pool), tag
    assert np.array_equal(valid.cpu().numpy(), o_valid), tag


@pytest.mark.parametrize("host_pool", [False, True])
def test_staging_golden(dev, host_pool):
    """Replay the reference's five-step trace (prefill chunks, decode,
    flushes, reuse of freed staging blocks)."""
    z = load_golden("tier_staging")
    L, NB, n_kv, d, page, NV, MAXF, steps = [int(x) for x in z["meta"]]
    stg = T.Staging(num_layers=L, num_blocks=NB, n_kv=n_kv, page=page, d=d,
                    max_reqs=3, max_pages=4, max_tokens=64, device=dev,
                    v_blocks=NV, max_flush=MAXF)
    if host_pool:
        hp = T.MappedHostVPool(num_layers=L, num_blocks=NB, n_kv=n_kv,
                               page=page, d=d, device=dev)
        pool_dev, pool_read = hp.dev_view, lambda: _i16(hp.host)
    else:
        pool_t = torch.zeros((L, NB, n_kv, page, d), dtype=torch.int16,
                             device=dev)
        pool_dev, pool_read = pool_t, lambda: pool_t.cpu().numpy()
    valid = torch.zeros((L, n_kv, NB), dtype=torch.int8, device=dev)
    bt = torch.from_numpy(z["block_table"]).to(dev)
    for s in range(steps):
        sl = z["steps_sl"][s]
        ql = z["steps_ql"][s]
        qsl = np.concatenate([[0], np.cumsum(ql)]).astype(np.int32)
        n_tok = int(qsl[-1])
        stg.begin_step(bt, torch.from_numpy(sl).to(dev),
                       torch.from_numpy(qsl).to(dev), int(ql.max()), n_tok,
                       pool=pool_dev, pool_valid=valid)
        vals = torch.from_numpy(z[f"vals_{s}"]).to(dev).view(torch.bfloat16)
        for l in range(L):
            stg.scatter_kv(l, None, vals[l], n_tok)
        torch.cuda.synchronize(dev)
        st = dict(vbo=z[f"vbo_{s}"], vfl=z[f"vfl_{s}"],
                  stack=z[f"stack_{s}"], top=int(z[f"top_{s}"][0]),
                  flist=z[f"flist_{s}"], fcnt=int(z[f"fcnt_{s}"][0]),
                  vslot=z[f"vslot_{s}"], v_pool=z[f"vpool_{s}"],
                  ovf=int(z[f"ovf_{s}"][0]))
        _check(stg, st, n_tok, pool_read(), valid, z[f"pool_{s}"],
               z[f"valid_{s}"], f"step {s}")
        stg.assert_free_partition()


def _random_steps(rng, R, MP, page, n_steps, chunk):
    """Per step: every request either idles (ql 0), decodes one token or
    takes a prefill chunk of up to ``chunk`` tokens, bounded by MP pages."""
    sl = np.zeros(R, np.int64)
    out = []
    for _ in range(n_steps):
        ql = np.zeros(R, np.int64)
        for r in range(R):
            room = MP * page - sl[r]
            if room <= 0:
                continue
            u = rng.random()
            if u < 0.15:
                continue
            ql[r] = 1 if (u < 0.6 and sl[r] > 0) else \
                int(rng.integers(1, chunk + 1))
            ql[r] = min(ql[r], room)
        sl = sl + ql
        out.append((sl.astype(np.int32).copy(), ql.astype(np.int32)))
    return out


@pytest.mark.parametrize("NV,MAXF,offload_k,d,cap", [
    (None, None, False, 128, 4096),  # default sizing: no overflow
    (None, None, True, 128, 4096),   # mem-kv: K staged and flushed beside V
    (14, 3, False, 64, 4096),        # flush-list cap (undo), stack underflow
    (None, None, False, 64, 0),      # collect walks every page (no pre-pass)
    (None, None, False, 64, 2),      # pre-pass list overflows on some steps
])
def test_staging_random_vs_oracle(dev, NV, MAXF, offload_k, d, cap):
    rng = np.random.default_rng(7 + (NV or 0) + d + offload_k + cap)
    L, R, MP, page, n_kv, chunk = 3, 6, 12, 16, 4, 40
    NB = R * MP + 9
    max_tokens = R * chunk
    stg = T.Staging(num_layers=L, num_blocks=NB, n_kv=n_kv, page=page, d=d,
                    max_reqs=R, max_pages=MP, max_tokens=max_tokens,
                    device=dev, v_blocks=NV, max_flush=MAXF,
                    offload_k=offload_k, cand_cap=cap)
    NVr, MAXFr = stg.NV, stg.MAXF
    bt_np = rng.permutation(NB)[:R * MP].astype(np.int32).reshape(R, MP)
    bt = torch.from_numpy(bt_np).to(dev)
    pool = torch.zeros((L, NB, n_kv, page, d), dtype=torch.int16, device=dev)
    poolk = torch.zeros_like(pool) if offload_k else None
    valid = torch.zeros((L, n_kv, NB), dtype=torch.int8, device=dev)
    sv = _oracle_state(L, NB, n_kv, d, page, NVr, MAXFr, max_tokens)
    sk = _oracle_state(L, NB, n_kv, d, page, NVr, MAXFr, max_tokens)
    o_pool = np.zeros((L, NB, n_kv, page, d), np.int16)
    o_poolk = np.zeros_like(o_pool)
    o_valid = np.zeros((L, n_kv, NB), np.int8)
    o_validk = np.zeros_like(o_valid)
    saw_flush = saw_ovf = False
    for s, (sl, ql) in enumerate(_random_steps(rng, R, MP, page, 24, chunk)):
        qsl = np.concatenate([[0], np.cumsum(ql)]).astype(np.int32)
        n_tok = int(qsl[-1])
        stg.begin_step(bt, torch.from_numpy(sl).to(dev),
                       torch.from_numpy(qsl).to(dev), int(ql.max()), n_tok,
                       pool=pool, pool_valid=valid, poolk=poolk)
        vals = rng.integers(-2**15, 2**15, (L, n_tok, n_kv, d), dtype=np.int16)
        keys = rng.integers(-2**15, 2**15, (L, n_tok, n_kv, d), dtype=np.int16)
        vd = torch.from_numpy(vals).to(dev).view(torch.bfloat16)
        kd = torch.from_numpy(keys).to(dev).view(torch.bfloat16)
        for l in range(L):
            stg.scatter_kv(l, kd[l] if offload_k else None, vd[l], n_tok)
        torch.cuda.synchronize(dev)
        O.staging_begin_step(sv, bt_np, sl, qsl, n_tok, page=page,
                             pool=o_pool, pool_valid=o_valid)
        for l in range(L):
            O.staging_scatter(sv, l, vals[l], n_tok, page=page)
        _check(stg, sv, n_tok, pool.cpu().numpy(), valid, o_pool, o_valid,
               f"step {s}")
        if offload_k:
            O.staging_begin_step(sk, bt_np, sl, qsl, n_tok, page=page,
                                 pool=o_poolk, pool_valid=o_validk)
            for l in range(L):
                O.staging_scatter(sk, l, keys[l], n_tok, page=page)
            assert np.array_equal(_i16(stg.k_pool), sk["v_pool"]), s
            assert np.array_equal(poolk.cpu().numpy(), o_poolk), s
        saw_flush |= sv["fcnt"] > 0
        saw_ovf |= sv["ovf"] > 0
        if not sv["ovf"]:
            stg.assert_free_partition()
    assert saw_flush
    if NV is not None:
        assert saw_ovf, "the undersized case must overflow"
