"""Generate golden vectors by running the REFERENCE's own kernels on CPU.

Run in a container that has the reference source tree (read-only) at
``$AMASS_REF_SRC`` (required; no default path):

    python tests/golden/make_golden.py

It imports the reference package with ``TRITON_INTERPRET=1`` (its Triton
kernels execute in the CPU interpreter), feeds it seeded inputs from
``amass_kv_b200.workloads`` and writes ``tests/golden/*.npz``: inputs plus the
reference outputs of derive_page_params, quad_score (+ nrm/max combine),
topb_select, sparse_paged_decode_batched (+ merge), r8_score, the residency
gather (exact LRU + fetch) and the ptr-select tiered decode.  The fixtures are
committed; nothing at test time reads the reference tree.

Coverage selection has no graph-safe reference (the reference's
``_nucleus_b`` is a scalar over heads, ``backend/_selection_bridge.py:117-133``);
its golden is ``_nucleus_b`` applied to each (request, kv-head) unit's masses
followed by the reference ``topb_select`` kernel run with that unit's b.
"""
from __future__ import annotations

import os
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"
os.environ.setdefault("AMASS_EIGH", "torch")
REF = os.environ.get("AMASS_REF_SRC")
if not REF:
    sys.exit("set AMASS_REF_SRC to the reference checkout's src/ directory")
HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, REF)

import numpy as np  # noqa: E402
import torch  # noqa: E402

from amass_kv_b200.workloads import (make_clse_case, make_quad_case,  # noqa: E402
                                     make_r8_case)

from amass.selection import (QuadState, R8State, derive_page_params,  # noqa
                             quad_score, r8_score, topb_select, clse_score)
from amass.attention.decode import (ResidentVSource,  # noqa: E402
                                    ensure_stage_b_buffers,
                                    sparse_paged_decode_batched)
from amass.backend._selection_bridge import _nucleus_b  # noqa: E402
from amass.tier.residency import Residency  # noqa: E402
from amass.selection.quad_build import quad_build_tail, quad_build_bulk  # noqa: E402
from amass.selection.build import _delta_select  # noqa: E402
from amass.tier.staging import Staging  # noqa: E402
from amass.tier.decode_mem import mem_decode_ptrsel  # noqa: E402


def t_bf16(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(
        torch.bfloat16)


def bf16_bits(t):
    return t.contiguous().view(torch.int16).numpy()


def kv_cache_of(case):
    """(NB, 2, page, n_kv, d) bf16 -- the vLLM 0.24 layout."""
    return torch.stack([t_bf16(case.K), t_bf16(case.V)], dim=1).contiguous()


def quad_state(case, *, budget, combine, n_req, sink=1, window=1):
    NB = case.K.shape[0]
    st = QuadState("cpu", num_layers=1, num_blocks=NB, n_kv=case.n_kv,
                   G=case.G, head_dim=case.d, page=case.page, max_reqs=n_req,
                   max_pages=case.MP, rank=case.r, budget=budget,
                   sink_pages=sink, window_pages=window, v_bits=case.v_bits,
                   combine=combine)
    st.quad_mu[0].copy_(torch.from_numpy(case.mu))
    st.mu_scale[0].copy_(torch.from_numpy(case.mu_s))
    st.quad_V[0].copy_(torch.from_numpy(case.Vq))
    st.V_scale[0].copy_(torch.from_numpy(case.V_s))
    st.quad_sig2[0].copy_(torch.from_numpy(case.sig2))
    st.score.fill_(float("nan"))
    if combine == "nrm":
        st.score_h.fill_(float("nan"))
    return st


def run_decode(case, st, q, kv, bt, sl, split=8):
    """The reference decode + merge.  The Triton CPU interpreter mis-evaluates
    ``tl.dot`` on bf16 operands, so q and the cache go in as float32 tensors
    holding the exact bf16 values (the kernel's fp16 P.V path is unchanged)."""
    st.D = case.d
    ensure_stage_b_buffers(st, "cpu", split)
    q, kv = q.float(), kv.float()
    out = torch.zeros(q.shape, dtype=torch.float32)
    sparse_paged_decode_batched(q, kv, bt, sl, st, out, ResidentVSource(kv),
                                scale=case.scale)
    return out


def quad_inputs(case):
    return dict(q=bf16_bits(t_bf16(case.q)),
                kv=bf16_bits(kv_cache_of(case)),
                block_table=case.block_table, seq_lens=case.seq_lens,
                mu=case.mu, mu_s=case.mu_s, Vq=case.Vq, V_s=case.V_s,
                sig2=case.sig2,
                meta=np.array([case.G, case.r, case.v_bits, case.page,
                               case.MP], dtype=np.int64),
                scale=np.array([case.scale], dtype=np.float64))


def gen_quad(name, case, *, budget, combine, coverage=None):
    n_req = case.block_table.shape[0]
    st = quad_state(case, budget=budget, combine=combine, n_req=n_req)
    q = t_bf16(case.q)
    bt = torch.from_numpy(case.block_table)
    sl = torch.from_numpy(case.seq_lens)
    kv = kv_cache_of(case)
    derive_page_params(st, sl, n_req)
    quad_score(st, 0, q, bt, sl, n_req, case.scale)
    res = dict(n_pages=st.n_pages.numpy().copy(),
               n_sel_hi=st.n_sel_hi.numpy().copy(),
               b_fix=st.b_fix.numpy().copy(), score=st.score.numpy().copy())
    if combine == "nrm":
        res["score_h"] = st.score_h.numpy().copy()
    if coverage is None:
        topb_select(st, n_req)
        res["page_table"] = st.page_table.numpy().copy()
        res["page_cnt"] = st.page_cnt.numpy().copy()
    else:
        # per-unit nucleus b via the reference _nucleus_b, then the reference
        # topb kernel with that b, one (request, kv-head) unit at a time.
        tab = np.full((n_req, case.n_kv, case.MP), -1, np.int32)
        cnt = np.zeros((n_req, case.n_kv), np.int32)
        bu = np.zeros((n_req, case.n_kv), np.int32)
        nsh = st.n_sel_hi.numpy().copy()
        b_saved = st.b_fix.clone()
        for rq in range(n_req):
            for kh in range(case.n_kv):
                n = int(nsh[rq])
                if n - 1 <= 1:
                    b = 1
                else:
                    sc = st.score[rq, kh, :n].double()
                    lm = sc.log() if combine == "nrm" else sc
                    b = _nucleus_b(lm[None, None, :], 1, n, coverage)
                bu[rq, kh] = b
                st.b_fix.copy_(b_saved)
                st.b_fix[rq] = b
                topb_select(st, n_req)
                tab[rq, kh] = st.page_table[rq, kh].numpy()
                cnt[rq, kh] = int(st.page_cnt[rq, kh])
        st.page_table.copy_(torch.from_numpy(tab))
        st.page_cnt.copy_(torch.from_numpy(cnt))
        res.update(page_table=tab, page_cnt=cnt, b_u=bu,
                   coverage=np.array([coverage]))
    out = run_decode(case, st, q, kv, bt, sl)
    res["out"] = out.float().numpy()
    np.savez_compressed(os.path.join(HERE, name + ".npz"),
                        budget=np.array([budget]),
                        combine=np.array([combine]),
                        **quad_inputs(case), **res)
    print(name, "cnt", res["page_cnt"].tolist())


def gen_r8(name, case, *, budget):
    n_req = case.block_table.shape[0]
    NB = case.K.shape[0]
    st = R8State("cpu", num_layers=1, num_blocks=NB, n_kv=case.K.shape[2],
                 G=case.G, head_dim=case.K.shape[3], page=case.page,
                 max_reqs=n_req, max_pages=case.MP, rank=case.r,
                 budget=budget, vk_bits=case.vk_bits, c_bits=case.c_bits)
    st.r8_mu[0].copy_(torch.from_numpy(case.mu))
    st.mu_scale[0].copy_(torch.from_numpy(case.mu_s))
    st.r8_Vk[0].copy_(torch.from_numpy(case.Vk))
    st.Vk_scale[0].copy_(torch.from_numpy(case.Vk_s))
    st.r8_c[0].copy_(torch.from_numpy(case.c))
    st.c_scale[0].copy_(torch.from_numpy(case.c_s))
    st.score.fill_(float("nan"))
    q = t_bf16(case.q)
    bt = torch.from_numpy(case.block_table)
    sl = torch.from_numpy(case.seq_lens)
    derive_page_params(st, sl, n_req)
    r8_score(st, 0, q, bt, sl, n_req, case.scale)
    topb_select(st, n_req)
    np.savez_compressed(
        os.path.join(HERE, name + ".npz"),
        q=bf16_bits(q), block_table=case.block_table, seq_lens=case.seq_lens,
        mu=case.mu, mu_s=case.mu_s, Vk=case.Vk, Vk_s=case.Vk_s, c=case.c,
        c_s=case.c_s,
        meta=np.array([case.G, case.r, case.vk_bits, case.c_bits, case.page,
                       case.MP, case.K.shape[2], case.K.shape[3]], np.int64),
        scale=np.array([case.scale]), budget=np.array([budget]),
        n_sel_hi=st.n_sel_hi.numpy(), n_pages=st.n_pages.numpy(),
        b_fix=st.b_fix.numpy(), score=st.score.numpy(),
        page_table=st.page_table.numpy(), page_cnt=st.page_cnt.numpy())
    print(name, "cnt", st.page_cnt.tolist())


def gen_clse(name, case, *, budget, combine):
    """The reference CLSE scorer (its default r'=2 path is the block-sweep
    kernel) + top-b on a quad case with per-token coordinates and resid."""
    n_req = case.block_table.shape[0]
    NB = case.K.shape[0]
    x = case.extra
    st = QuadState("cpu", num_layers=1, num_blocks=NB, n_kv=case.n_kv,
                   G=case.G, head_dim=case.d, page=case.page, max_reqs=n_req,
                   max_pages=case.MP, rank=case.r, budget=budget,
                   v_bits=case.v_bits, combine=combine, coords="lse",
                   c_bits=x["c_bits"], c_grain=x["c_grain"])
    st.quad_mu[0].copy_(torch.from_numpy(case.mu))
    st.mu_scale[0].copy_(torch.from_numpy(case.mu_s))
    st.quad_V[0].copy_(torch.from_numpy(case.Vq))
    st.V_scale[0].copy_(torch.from_numpy(case.V_s))
    st.quad_sig2[0].copy_(torch.from_numpy(case.sig2))
    st.quad_c[0].copy_(torch.from_numpy(x["c"]))
    st.c_scale[0].copy_(torch.from_numpy(x["c_s"]))
    st.quad_resid[0].copy_(torch.from_numpy(x["resid"]))
    st.score.fill_(float("nan"))
    if combine == "nrm":
        st.score_h.fill_(float("nan"))
    q = t_bf16(case.q)
    bt = torch.from_numpy(case.block_table)
    sl = torch.from_numpy(case.seq_lens)
    derive_page_params(st, sl, n_req)
    clse_score(st, 0, q, bt, sl, n_req, case.scale)
    topb_select(st, n_req)
    extra = {}
    if combine == "nrm":
        extra["score_h"] = st.score_h.numpy()
    np.savez_compressed(
        os.path.join(HERE, name + ".npz"), **quad_inputs(case),
        c=x["c"], c_s=x["c_s"], resid=x["resid"],
        cmeta=np.array([x["c_bits"], 1 if x["c_grain"] == "token" else 0],
                       np.int64),
        combine=np.array([combine]), budget=np.array([budget]),
        n_sel_hi=st.n_sel_hi.numpy(), n_pages=st.n_pages.numpy(),
        b_fix=st.b_fix.numpy(), score=st.score.numpy(),
        page_table=st.page_table.numpy(), page_cnt=st.page_cnt.numpy(),
        **extra)
    print(name, "cnt", st.page_cnt.tolist())


def gen_build(name, *, seed, n_req, n_kv, d, ctxs, L, r, v_bits, coords,
              c_bits=4, c_grain="token"):
    """The reference's batched tail rebuild (quad_build_tail: the last
    finalized page of every request, every layer) on seeded K caches."""
    rng = np.random.default_rng(seed)
    page = 16
    npg = [(c + page - 1) // page for c in ctxs]
    NB = sum(npg) + 4
    perm = rng.permutation(NB).astype(np.int32)
    MP = max(npg)
    bt = np.zeros((n_req, MP), np.int32)
    o = 0
    for i, n in enumerate(npg):
        bt[i, :n] = perm[o:o + n]
        o += n
    K = rng.standard_normal((L, NB, page, n_kv, d)).astype(np.float32)
    K[:, :, :, :, :3] *= 4.0                                  # anisotropy
    Kb = t_bf16(K)
    st = QuadState("cpu", num_layers=L, num_blocks=NB, n_kv=n_kv, G=4,
                   head_dim=d, page=page, max_reqs=n_req, max_pages=MP,
                   rank=r, budget=0.1, v_bits=v_bits, coords=coords,
                   c_bits=c_bits, c_grain=c_grain)
    sl = torch.tensor(ctxs, dtype=torch.int32)
    n = quad_build_tail(st, [Kb[l] for l in range(L)],
                        torch.from_numpy(bt), sl, n_req)
    extra = {}
    if coords == "lse":
        extra = dict(c=st.quad_c.numpy(), c_s=st.c_scale.numpy(),
                     resid=st.quad_resid.numpy())
    np.savez_compressed(
        os.path.join(HERE, name + ".npz"), K=bf16_bits(Kb), block_table=bt,
        seq_lens=np.asarray(ctxs, np.int32),
        meta=np.array([L, NB, n_kv, d, r, v_bits, c_bits,
                       1 if c_grain == "token" else 0,
                       1 if coords == "lse" else 0], np.int64),
        mu=st.quad_mu.numpy(), mu_s=st.mu_scale.numpy(),
        V=st.quad_V.numpy(), V_s=st.V_scale.numpy(),
        sig2=st.quad_sig2.numpy(), tag=bf16_bits(st.quad_tag), **extra)
    print(name, "pages built", n)


STAGING_STEPS = [
    # (seq_lens after the step, new tokens per request) for 3 requests
    ([40, 20, 0], [40, 20, 0]),        # two prefills
    ([41, 35, 0], [1, 15, 0]),         # decode + second prefill chunk
    ([42, 36, 18], [1, 1, 18]),        # decodes + a new prefill
    ([48, 37, 19], [6, 1, 1]),         # a 6-token step crossing a page
    ([49, 48, 20], [1, 11, 1]),        # completes pages of request 1
]


def gen_staging(name, *, seed=31, L=2, NB=40, n_kv=2, d=64, page=16,
                v_blocks=12, max_flush=6):
    """The reference Staging.begin_step + scatter_kv over STAGING_STEPS."""
    rng = np.random.default_rng(seed)
    R = 3
    MP = 4
    bt = np.zeros((R, MP), np.int32)
    perm = rng.permutation(NB).astype(np.int32)
    bt[:] = perm[:R * MP].reshape(R, MP)
    stg = Staging(num_layers=L, num_blocks=NB, n_kv=n_kv, page=page, d=d,
                  max_reqs=R, max_pages=MP, max_tokens=64,
                  dtype=torch.bfloat16, device="cpu", v_blocks=v_blocks,
                  max_flush=max_flush)
    pool = torch.zeros((L, NB, n_kv, page, d), dtype=torch.int16)
    pool_valid = torch.zeros((L, n_kv, NB), dtype=torch.int8)
    rec = {}
    for s_, (sl, ql) in enumerate(STAGING_STEPS):
        qsl = np.concatenate([[0], np.cumsum(ql)]).astype(np.int32)
        n_tok = int(qsl[-1])
        slt = torch.tensor(sl, dtype=torch.int32)
        qslt = torch.from_numpy(qsl)
        stg.begin_step(torch.from_numpy(bt), slt, qslt, max(ql), n_tok,
                       pool=pool.view(-1), pool_valid=pool_valid)
        vals = t_bf16(rng.standard_normal((L, n_tok, n_kv, d)))
        for l in range(L):
            stg.scatter_kv(l, None, vals[l], n_tok)
        rec[f"vals_{s_}"] = bf16_bits(vals)
        rec[f"vbo_{s_}"] = stg.vbo.numpy().copy()
        rec[f"vfl_{s_}"] = stg.v_flushed.numpy().copy()
        rec[f"top_{s_}"] = stg.v_free_top.numpy().copy()
        rec[f"stack_{s_}"] = stg.v_free_stack.numpy().copy()
        rec[f"fcnt_{s_}"] = stg.flush_cnt.numpy().copy()
        rec[f"flist_{s_}"] = stg.flush_list.numpy().copy()
        rec[f"vslot_{s_}"] = stg.v_slot_mapping[:n_tok].numpy().copy()
        rec[f"pool_{s_}"] = pool.numpy().copy()
        rec[f"valid_{s_}"] = pool_valid.numpy().copy()
        rec[f"vpool_{s_}"] = bf16_bits(stg.v_pool).copy()
        rec[f"ovf_{s_}"] = stg.overflow.numpy().copy()
    np.savez_compressed(
        os.path.join(HERE, name + ".npz"), block_table=bt,
        meta=np.array([L, NB, n_kv, d, page, v_blocks, max_flush,
                       len(STAGING_STEPS)], np.int64),
        steps_sl=np.array([x[0] for x in STAGING_STEPS], np.int32),
        steps_ql=np.array([x[1] for x in STAGING_STEPS], np.int32), **rec)
    print(name, "final top", int(stg.v_free_top), "ovf", int(stg.overflow))


def gen_delta(name, *, seed=41, n_req=3, n_kv=2, d=64, L=2):
    """The reference's content-tag staleness pass (_delta_select) after a
    bulk build, once the keys of some blocks changed: in a tag channel of
    the page-final token (stale), in a non-tag channel (not stale), and one
    tag reset to NaN (stale)."""
    rng = np.random.default_rng(seed)
    page, ctxs = 16, [70, 130, 41]
    npg = [(c + page - 1) // page for c in ctxs]
    NB = sum(npg) + 3
    perm = rng.permutation(NB).astype(np.int32)
    MP = max(npg)
    bt = np.zeros((n_req, MP), np.int32)
    o = 0
    for i, n in enumerate(npg):
        bt[i, :n] = perm[o:o + n]
        o += n
    Kb = t_bf16(rng.standard_normal((L, NB, page, n_kv, d)).astype(np.float32))
    st = QuadState("cpu", num_layers=L, num_blocks=NB, n_kv=n_kv, G=4,
                   head_dim=d, page=page, max_reqs=n_req, max_pages=MP,
                   rank=2, budget=0.1, v_bits=4)
    sl = torch.tensor(ctxs, dtype=torch.int32)
    max_fin = max(c // page for c in ctxs)
    quad_build_bulk(st, [Kb[l] for l in range(L)], torch.from_numpy(bt), sl,
                    n_req, max_fin)
    fin = [bt[r, p] for r in range(n_req) for p in range(ctxs[r] // page)]
    pick = rng.choice(fin, 5, replace=False)
    Kb[1, pick[0], page - 1, 1, 2] += 1.0        # tag channel, layer 1
    Kb[0, pick[1], page - 1, 0, 0] += 1.0        # tag channel, layer 0
    Kb[0, pick[2], page - 1, 0, 40] += 1.0       # not a tag channel
    Kb[1, pick[3], 3, 1, 1] += 1.0               # not the page-final token
    st.quad_tag[0, pick[4], 1, 5] = float("nan")
    stale = _delta_select(st.quad_tag, [Kb[l] for l in range(L)],
                          torch.from_numpy(bt), sl, n_req, page, max_fin,
                          st.tagw)
    np.savez_compressed(
        os.path.join(HERE, name + ".npz"), K=bf16_bits(Kb),
        tag=bf16_bits(st.quad_tag), block_table=bt,
        seq_lens=np.array(ctxs, np.int32), max_fin=np.array([max_fin]),
        stale=stale.numpy().astype(np.int32))
    print(name, "stale", stale.tolist(), "picked", pick.tolist())


def gen_tier(name, case, *, budget, hot_slots=10, steps=3, seed=5):
    """Residency gather over several steps with forced eviction, staged and
    flushed sources, then the ptr-select tiered decode."""
    rng = np.random.default_rng(seed)
    n_req = case.block_table.shape[0]
    NB, page, n_kv, d = case.K.shape
    st = quad_state(case, budget=budget, combine="max", n_req=n_req)
    q = t_bf16(case.q)
    bt = torch.from_numpy(case.block_table)
    sl = torch.from_numpy(case.seq_lens)
    kv = kv_cache_of(case)
    derive_page_params(st, sl, n_req)
    res = Residency(num_layers=1, num_blocks=NB, n_kv=n_kv,
                    hot_slots=hot_slots, page=page, d=d, max_reqs=n_req,
                    max_pages=case.MP, dtype=torch.bfloat16, device="cpu")
    # pinned-pool stand-in (int16 bits), staging pool + vbo
    Vb = t_bf16(case.V)                                   # (NB, page, kv, d)
    pool = Vb.permute(0, 2, 1, 3).contiguous().view(torch.int16)[None].clone()
    NV = 6
    v_pool = torch.zeros((1, NV, page, n_kv, d), dtype=torch.bfloat16)
    vbo = torch.full((NB,), -1, dtype=torch.int32)
    staged = rng.choice(NB, NV, replace=False)
    for i, blk in enumerate(staged):
        vbo[blk] = i
        v_pool[0, i] = Vb[blk]
        pool[0, blk] = 0                                  # not flushed yet
    res.pool_valid.fill_(1)
    res.pool_valid[0, :, torch.from_numpy(staged)] = 0
    staging = types.SimpleNamespace(v_pool=v_pool, vbo=vbo, k_pool=None)
    tier = types.SimpleNamespace(residency=res, staging=staging,
                                 offload_k=False,
                                 pool=types.SimpleNamespace(dev_view=pool[0]
                                                            .view(-1)))
    rec = dict(staged=staged.astype(np.int32), NV=np.array([NV]),
               hot_slots=np.array([hot_slots]))
    pool_init = pool.clone()
    valid_init = res.pool_valid.clone()
    for s in range(steps):
        qs = t_bf16(case.q + 1.5 * s * rng.standard_normal(case.q.shape))
        quad_score(st, 0, qs, bt, sl, n_req, case.scale)
        topb_select(st, n_req)
        rec[f"q_{s}"] = bf16_bits(qs)
        rec[f"page_table_{s}"] = st.page_table.numpy().copy()
        rec[f"page_cnt_{s}"] = st.page_cnt.numpy().copy()
        res.gather(0, st.page_table, st.page_cnt, bt, sl, n_req, staging,
                   pool[0].view(-1))
        rec[f"page2slot_{s}"] = res.page2slot[0].numpy().copy()
        rec[f"slot2page_{s}"] = res.slot2page[0].numpy().copy()
        rec[f"lru_{s}"] = res.lru_clock[0].numpy().copy()
        rec[f"hot_{s}"] = res.hot_i16[0].numpy().copy()
        rec[f"pool_valid_{s}"] = res.pool_valid[0].numpy().copy()
        rec[f"fetch_cnt_{s}"] = res.fetch_cnt.numpy().copy()
        rec[f"overflow_{s}"] = res.overflow.numpy().copy()
        st.D = d
        ensure_stage_b_buffers(st, "cpu", 8)
        out = torch.zeros(qs.shape, dtype=torch.float32)
        mem_decode_ptrsel(qs.float(), kv.float(), bt, sl, st, out, tier, 0,
                          scale=case.scale)
        rec[f"out_{s}"] = out.float().numpy()
        out2 = run_decode(case, st, qs, kv, bt, sl)
        rec[f"out_resident_{s}"] = out2.float().numpy()
        print(name, "step", s, "fetch", int(res.fetch_cnt), "ovf",
              int(res.overflow))
    np.savez_compressed(os.path.join(HERE, name + ".npz"),
                        **quad_inputs(case), budget=np.array([budget]),
                        pool_init=pool_init.numpy(),
                        pool_valid_init=valid_init[0].numpy(),
                        v_pool=bf16_bits(v_pool), vbo=vbo.numpy(),
                        pool_final=pool.numpy(), steps=np.array([steps]),
                        **rec)


def gen_invalidate(name, *, seed=9, L=2, n_kv=2, NB=40, S=12, page=16):
    """Residency.invalidate_written on a populated residency: random maps
    and validity, requests that appended 1 or several tokens (chunked
    prefill), one empty request."""
    rng = np.random.default_rng(seed)
    res = Residency(num_layers=L, num_blocks=NB, n_kv=n_kv, hot_slots=S,
                    page=page, d=64, max_reqs=4, max_pages=8,
                    dtype=torch.bfloat16, device="cpu")
    for l in range(L):
        for kv in range(n_kv):
            blks = rng.choice(NB, S, replace=False)
            for s_, b in enumerate(blks):
                if rng.random() < 0.8:
                    res.page2slot[l, kv, b] = s_
                    res.slot2page[l, kv, s_] = b
    res.pool_valid.copy_(torch.from_numpy(
        (rng.random((L, n_kv, NB)) < 0.7).astype(np.int8)))
    bt = torch.from_numpy(rng.permutation(NB)[:32].reshape(4, 8)
                          .astype(np.int32))
    sl = torch.tensor([100, 33, 0, 128], dtype=torch.int32)
    qsl = torch.tensor([0, 1, 21, 21, 61], dtype=torch.int32)
    p2s0 = res.page2slot.numpy().copy()
    s2p0 = res.slot2page.numpy().copy()
    v0 = res.pool_valid.numpy().copy()
    res.invalidate_written(bt, sl, qsl)
    np.savez_compressed(os.path.join(HERE, name + ".npz"),
                        block_table=bt.numpy(), seq_lens=sl.numpy(),
                        query_start_loc=qsl.numpy(), page=np.array([page]),
                        page2slot_init=p2s0, slot2page_init=s2p0,
                        pool_valid_init=v0,
                        page2slot=res.page2slot.numpy(),
                        slot2page=res.slot2page.numpy(),
                        pool_valid=res.pool_valid.numpy())
    print(name, "cleared", int((p2s0 >= 0).sum() - (res.page2slot >= 0).sum()
                              .item()))


def main():
    torch.manual_seed(0)
    # C1: B=2, 8 q / 2 kv heads, d=64, ctx 2048, r'=8 int8 V, budget 0.10, nrm
    c1 = make_quad_case(0, n_req=2, n_kv=2, G=4, d=64, ctxs=(2048, 2048),
                        r=8, v_bits=8, heavy=4, shift=2.0)
    gen_quad("quad_c1_nrm", c1, budget=0.10, combine="nrm")
    gen_quad("quad_c1_max", c1, budget=0.10, combine="max")
    # Llama geometry slice: d=128, G=4, r'=2 int4 V; ragged incl. a 1-page,
    # a 2-page (keep-all) and an empty (seq_len 0) request.
    c2 = make_quad_case(1, n_req=5, n_kv=2, G=4, d=128,
                        ctxs=(1000, 517, 16, 20, 0), r=2, v_bits=4, heavy=3,
                        shift=3.0, outlier_frac=0.02)
    gen_quad("quad_d128_i4_nrm", c2, budget=0.2, combine="nrm")
    gen_quad("quad_d128_i4_max", c2, budget=0.05, combine="max")
    gen_quad("quad_d128_i4_cov", c2, budget=0.1, combine="nrm",
             coverage=0.9)
    c3 = make_quad_case(2, n_req=2, n_kv=2, G=8, d=128, ctxs=(700, 333),
                        r=2, v_bits=8, heavy=3, shift=3.0)
    gen_quad("quad_g8_i8_cov_max", c3, budget=0.1, combine="max",
             coverage=0.95)
    r8a = make_r8_case(3, n_req=2, n_kv=2, G=4, d=64, ctxs=(1024, 700), r=8)
    gen_r8("r8_i8", r8a, budget=0.1)
    r8b = make_r8_case(4, n_req=2, n_kv=2, G=4, d=128, ctxs=(600, 250), r=8,
                       vk_bits=4, c_bits=4)
    gen_r8("r8_i4", r8b, budget=0.1)
    t = make_quad_case(6, n_req=2, n_kv=2, G=4, d=64, ctxs=(500, 301),
                       r=2, v_bits=8, heavy=3, shift=2.5)
    gen_tier("tier_lru", t, budget=0.25, hot_slots=24, steps=3)
    gen_tier("tier_overflow", t, budget=0.25, hot_slots=10, steps=1)
    gen_invalidate("tier_invalidate")
    cl1 = make_clse_case(7, n_req=2, n_kv=2, G=4, d=64, ctxs=(700, 333), r=2,
                         v_bits=4, c_bits=4, c_grain="token")
    gen_clse("clse_i4_tok_nrm", cl1, budget=0.1, combine="nrm")
    cl2 = make_clse_case(8, n_req=3, n_kv=2, G=8, d=128, ctxs=(900, 260, 40),
                         r=2, v_bits=8, c_bits=8, c_grain="page")
    gen_clse("clse_i8_page_max", cl2, budget=0.1, combine="max")
    cl3 = make_clse_case(9, n_req=2, n_kv=2, G=4, d=128, ctxs=(500, 377),
                         r=4, v_bits=8, c_bits=8, c_grain="token")
    gen_clse("clse_r4_i8_tok_max", cl3, budget=0.1, combine="max")
    gen_staging("tier_staging")
    gen_delta("build_delta_tags")
    gen_build("build_quad_i4", seed=21, n_req=3, n_kv=2, d=128,
              ctxs=[100, 257, 16], L=2, r=2, v_bits=4, coords="none")
    gen_build("build_clse_i8", seed=22, n_req=2, n_kv=2, d=64,
              ctxs=[300, 48], L=2, r=4, v_bits=8, coords="lse", c_bits=8,
              c_grain="page")


if __name__ == "__main__":
    main()
