"""Serving wiring of the mem tier (MemSession): an engine-style run of
chunked prefill steps followed by many decode steps, with K written to the
K-only cache at the engine's slot mapping, V through staging / flush / the
pinned pool, a hot buffer small enough to evict, summaries refreshed as
pages complete, and on every pure-decode step the tiered decode of every
layer compared with the resident decode of a full K+V cache holding the
same tokens under the same selection.

Bar (the reference's system gate, tier/README.md): bitwise equal outputs on
every decode step and layer; tier invariants hold after every step.
"""
import numpy as np
import pytest
import torch

from amass_kv_b200 import attention as A
from amass_kv_b200 import summaries as SM
from amass_kv_b200.serving import MemSession

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _steps(rng, R, cap, n_prefill, n_decode, chunk):
    sl = np.zeros(R, np.int64)
    out = []
    for s in range(n_prefill + n_decode):
        if s < n_prefill:
            ql = rng.integers(1, chunk + 1, R)
        else:
            ql = np.ones(R, np.int64)
        ql = np.minimum(ql, cap - sl)
        sl = sl + ql
        out.append((sl.astype(np.int32), ql.astype(np.int32)))
    return out


@pytest.mark.parametrize("offload_k,scorer", [(False, "quad"), (True, "quad"),
                                              (False, "clse")])
def test_mem_session_bitwise_equals_resident(dev, offload_k, scorer):
    rng = np.random.default_rng(3 + offload_k)
    L, R, MP, page, n_kv, G, d = 2, 3, 24, 16, 2, 4, 128
    NB = R * MP + 7
    chunk = 70
    sess = MemSession(num_layers=L, num_blocks=NB, n_kv=n_kv, G=G,
                      head_dim=d, max_reqs=R, max_pages=MP,
                      max_tokens=R * chunk, page=page, hot_slots=20,
                      budget=0.3, offload_k=offload_k, device=dev,
                      scorer=scorer)
    bt_np = rng.permutation(NB)[:R * MP].astype(np.int32).reshape(R, MP)
    bt = torch.from_numpy(bt_np).to(dev)
    kv_full = torch.zeros((L, NB, 2, page, n_kv, d), dtype=torch.bfloat16,
                          device=dev)
    scale = d ** -0.5
    decoded = 0
    for s, (sl, ql) in enumerate(_steps(rng, R, MP * page, 3, 40, chunk)):
        qsl = np.concatenate([[0], np.cumsum(ql)]).astype(np.int32)
        n_tok = int(qsl[-1])
        pos = np.concatenate([np.arange(sl[r] - ql[r], sl[r])
                              for r in range(R)])
        req = np.repeat(np.arange(R), ql)
        slots = torch.from_numpy(bt_np[req, pos // page].astype(np.int64) * page
                                 + pos % page).to(dev)
        sl_t = torch.from_numpy(sl).to(dev)
        qsl_t = torch.from_numpy(qsl).to(dev)
        sess.begin_step(bt, sl_t, qsl_t, int(ql.max()), n_tok)
        for l in range(L):
            k = torch.randn((n_tok, n_kv, d), device=dev).to(torch.bfloat16)
            v = torch.randn((n_tok, n_kv, d), device=dev).to(torch.bfloat16)
            sess.write_kv(l, k, v, slots, n_tok)
            blk, off = slots // page, slots % page
            kv_full[l, blk, 0, off] = k
            kv_full[l, blk, 1, off] = v
        if offload_k:
            SM.quad_build_tail(sess.st, [kv_full[l][:, 0] for l in range(L)],
                               bt, sl_t, R)
        else:
            sess.refresh_summaries()
        sess.tier.assert_invariants(bt, sl_t, qsl_t)
        if not (ql == 1).all():
            continue
        for l in range(L):
            q = torch.randn((R, n_kv * G, d), device=dev).to(torch.bfloat16)
            out = torch.zeros_like(q)
            sess.decode(l, q, out, scale=scale)
            ref = torch.zeros_like(q)
            A.sparse_paged_decode_batched_cuda(q, kv_full[l], bt, sl_t,
                                               sess.st, ref, scale=scale)
            torch.cuda.synchronize(dev)
            assert torch.equal(out, ref), (s, l)
            assert int(sess.st.page_cnt.min()) > 0
        decoded += 1
    assert decoded >= 30
    # the hot buffer was too small for the working set: pages were evicted
    # and fetched again from the pinned pool
    assert int(sess.tier.residency.clock[0]) > decoded
    vb = sess.vram_bytes()
    assert vb["k_cache"] < vb["resident_kv_equivalent"]


def test_forward_mem_seam(dev):
    """The reference's attention seam driven as vLLM drives it, without
    model weights: per step the builder half (begin_step_from_metadata)
    runs once, then every layer calls forward_mem(layer, query, key, value,
    kv_cache, attn_metadata, output) with the reference's argument list
    (backend/attn.py:85-120); the layer is found from its cache address.
    Pure-decode outputs are bitwise equal to the resident decode of a full
    K+V cache; prefill steps return None (the engine's attention runs)."""
    from types import SimpleNamespace
    rng = np.random.default_rng(17)
    L, R, MP, page, n_kv, G, d = 2, 3, 16, 16, 2, 4, 128
    NB = R * MP + 5
    sess = MemSession(num_layers=L, num_blocks=NB, n_kv=n_kv, G=G,
                      head_dim=d, max_reqs=R, max_pages=MP,
                      max_tokens=R * 64, page=page, hot_slots=16, budget=0.3,
                      device=dev)
    k_caches = [sess.k_cache[l] for l in range(L)]
    sess.bind_kv_caches(k_caches)
    bt_np = rng.permutation(NB)[:R * MP].astype(np.int32).reshape(R, MP)
    bt = torch.from_numpy(bt_np).to(dev)
    kv_full = torch.zeros((L, NB, 2, page, n_kv, d), dtype=torch.bfloat16,
                          device=dev)
    scale = d ** -0.5
    decoded = 0
    for s, (sl, ql) in enumerate(_steps(rng, R, MP * page, 2, 12, 64)):
        qsl = np.concatenate([[0], np.cumsum(ql)]).astype(np.int32)
        n_tok = int(qsl[-1])
        pos = np.concatenate([np.arange(sl[r] - ql[r], sl[r])
                              for r in range(R)])
        req = np.repeat(np.arange(R), ql)
        slots = torch.from_numpy(bt_np[req, pos // page].astype(np.int64) *
                                 page + pos % page).to(dev)
        m = SimpleNamespace(block_table=bt, seq_lens=torch.from_numpy(sl).to(dev),
                            query_start_loc=torch.from_numpy(qsl).to(dev),
                            max_query_len=int(ql.max()),
                            num_actual_tokens=n_tok, slot_mapping=slots)
        sess.begin_step_from_metadata(m)
        for l in range(L):
            k = torch.randn((n_tok, n_kv, d), device=dev).to(torch.bfloat16)
            v = torch.randn((n_tok, n_kv, d), device=dev).to(torch.bfloat16)
            q = torch.randn((n_tok, n_kv * G, d), device=dev).to(torch.bfloat16)
            out = torch.zeros((n_tok, n_kv * G * d), dtype=torch.bfloat16,
                              device=dev)
            got = sess.forward_mem(SimpleNamespace(), q, k, v, k_caches[l], m,
                                   out, None, None, scale=scale)
            blk, off = slots // page, slots % page
            kv_full[l, blk, 0, off] = k
            kv_full[l, blk, 1, off] = v
            if m.max_query_len != 1:
                assert got is None
                continue
            ref = torch.zeros((R, n_kv * G, d), dtype=torch.bfloat16,
                              device=dev)
            A.sparse_paged_decode_batched_cuda(q, kv_full[l], bt, m.seq_lens,
                                               sess.st, ref, scale=scale)
            torch.cuda.synchronize(dev)
            assert got is out
            assert torch.equal(out.view(R, n_kv * G, d), ref), (s, l)
            decoded += 1
        sess.refresh_summaries()
    assert decoded >= 20
