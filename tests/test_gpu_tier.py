"""GPU parity of the mem-v / mem-kv tier: residency plan, miss fetch from the
pinned mapped host pool, invalidation and the ptr-select decode, through the
C ABI, against the reference's golden residency traces and the CPU oracle.

Bars: residency maps, LRU clocks, pool validity, fetch counts, overflow and
every copied byte are bit-exact; the tiered decode is bitwise equal to the
resident decode over the same bytes, and within bf16 tolerance (2e-2 abs,
1e-2 rel) of the reference's fp32 output.
"""
import numpy as np
import pytest
import torch

from amass_kv_b200 import attention as A
from amass_kv_b200 import tier as T
from amass_kv_b200.selection import QuadState
from oracle import amass_oracle as O
from tests.conftest import bits_to_f32, load_golden

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _bits(t):
    return t.view(torch.int16).cpu().numpy()


def _state(dev, *, n_req, n_kv, G, d, NB, MP):
    st = QuadState(dev, num_layers=1, num_blocks=NB, n_kv=n_kv, G=G,
                   head_dim=d, page=16, max_reqs=n_req, max_pages=MP, rank=2,
                   budget=0.1, v_bits=8, combine="max")
    A.ensure_stage_b_buffers(st, dev, 128)
    return st


@pytest.mark.parametrize("name", ["tier_lru", "tier_overflow"])
def test_tier_golden_trace(name, dev):
    """Replay the reference's residency trace (its selections, its pools):
    maps, clocks, validity, hot bytes, write-through and outputs."""
    z = load_golden(name)
    kv_bits = z["kv"]                               # (NB, 2, page, n_kv, d)
    NB, _, page, n_kv, d = kv_bits.shape
    G = int(z["meta"][0])
    MP = int(z["meta"][4])
    S = int(z["hot_slots"][0])
    n_req = z["block_table"].shape[0]
    tier = T.Tier(num_layers=1, num_blocks=NB, n_kv=n_kv, page=page, d=d,
                  hot_slots=S, max_reqs=n_req, max_pages=MP,
                  n_vslots=int(z["NV"][0]), device=dev)
    tier.pool.host.view(torch.int16).copy_(torch.from_numpy(z["pool_init"]))
    r5 = tier.residency
    r5.pool_valid[0].copy_(torch.from_numpy(z["pool_valid_init"]))
    tier.staging.v_pool.view(torch.int16).copy_(torch.from_numpy(z["v_pool"]))
    tier.staging.vbo.copy_(torch.from_numpy(z["vbo"]))
    kv = torch.from_numpy(kv_bits).view(torch.bfloat16).to(dev)
    bt = torch.from_numpy(z["block_table"]).to(dev)
    sl = torch.from_numpy(z["seq_lens"]).to(dev)
    st = _state(dev, n_req=n_req, n_kv=n_kv, G=G, d=d, NB=NB, MP=MP)
    scale = float(z["scale"][0])
    for s in range(int(z["steps"][0])):
        st.page_table.copy_(torch.from_numpy(z[f"page_table_{s}"]))
        st.page_cnt.copy_(torch.from_numpy(z[f"page_cnt_{s}"]))
        q = torch.from_numpy(z[f"q_{s}"]).view(torch.bfloat16).to(dev)
        out = torch.zeros(q.shape, dtype=torch.bfloat16, device=dev)
        T.mem_dynamic_decode(q, kv, bt, sl, st, out, tier, 0, scale=scale)
        res = torch.zeros_like(out)
        A.sparse_paged_decode_batched_cuda(q, kv, bt, sl, st, res, scale=scale)
        torch.cuda.synchronize()
        assert np.array_equal(r5.page2slot[0].cpu().numpy(), z[f"page2slot_{s}"])
        assert np.array_equal(r5.slot2page[0].cpu().numpy(), z[f"slot2page_{s}"])
        assert np.array_equal(r5.lru_clock[0].cpu().numpy(), z[f"lru_{s}"])
        assert np.array_equal(r5.pool_valid[0].cpu().numpy(),
                              z[f"pool_valid_{s}"])
        assert r5.misses_last_call() == int(z[f"fetch_cnt_{s}"][0])
        assert int(r5.overflow[0]) == int(z[f"overflow_{s}"][0])
        s2p = z[f"slot2page_{s}"]
        hot = _bits(r5.hot[0])
        for k in range(n_kv):
            for slot in range(S):
                if s2p[k, slot] >= 0:
                    assert np.array_equal(hot[k, slot], z[f"hot_{s}"][k, slot])
        o = out.float().cpu().numpy()
        np.testing.assert_allclose(o, z[f"out_{s}"], atol=ATOL, rtol=RTOL)
        if name == "tier_lru":
            # every V byte the tier serves equals the resident cache's
            assert torch.equal(out, res)
    r5.assert_maps_inverse()
    assert np.array_equal(tier.pool.host.view(torch.int16).numpy(),
                          z["pool_final"])


def _random_tier_case(seed, *, n_req, n_kv, G, d, S, steps, L=2, layer=1,
                      mem_kv=False, invalidate=False):
    rng = np.random.default_rng(seed)
    page = 16
    ctx = rng.integers(40, 900, n_req)
    ctx[0] = max(ctx[0], 300)
    npg = -(-ctx // page)
    MP = int(npg.max())
    share = 4                                  # shared prefix blocks
    NB = int(npg.sum()) + 8
    perm = rng.permutation(NB)
    bt = np.zeros((n_req, MP), np.int32)
    nxt = 0
    for r in range(n_req):
        for p in range(npg[r]):
            if r > 0 and p < share and npg[r] > share:
                bt[r, p] = bt[0, p]
            else:
                bt[r, p] = perm[nxt]
                nxt += 1
    K = rng.standard_normal((NB, page, n_kv, d)).astype(np.float32)
    V = rng.standard_normal((NB, page, n_kv, d)).astype(np.float32)
    K, V = O.bf16_round(K), O.bf16_round(V)
    sels = []
    for s in range(steps):
        tab = np.full((n_req, n_kv, MP), -1, np.int32)
        cnt = np.zeros((n_req, n_kv), np.int32)
        for r in range(n_req):
            for k in range(n_kv):
                b = int(rng.integers(1, max(2, npg[r] // 3)))
                # drift: half the selection stays near the previous centre
                pages = np.unique(np.concatenate([
                    rng.choice(npg[r], min(b, npg[r]), replace=False),
                    [npg[r] - 1]]))
                tab[r, k, :len(pages)] = pages
                cnt[r, k] = len(pages)
        sels.append((tab, cnt))
    return dict(rng=rng, page=page, ctx=ctx.astype(np.int32), MP=MP, NB=NB,
                bt=bt, K=K, V=V, sels=sels, L=L, layer=layer, n_kv=n_kv, G=G,
                d=d, S=S, n_req=n_req, mem_kv=mem_kv, invalidate=invalidate)


@pytest.mark.parametrize("seed,n_req,n_kv,G,d,S,mem_kv,inval,fetch", [
    (0, 4, 2, 4, 128, 40, False, False, "kernel"),
    (1, 6, 4, 8, 64, 24, False, True, "kernel"),
    (2, 3, 2, 4, 128, 6, False, False, "kernel"),  # overflow: S below a step
    (3, 5, 2, 4, 128, 64, True, True, "kernel"),   # mem-kv
    (4, 8, 8, 4, 128, 300, False, False, "kernel"),
    (0, 4, 2, 4, 128, 40, False, False, "dma"),    # copy engines + staged kernel
    (3, 5, 2, 4, 128, 64, True, True, "dma"),      # mem-kv over copy engines
])
def test_tier_random_vs_oracle(seed, n_req, n_kv, G, d, S, mem_kv, inval,
                               fetch, dev):
    c = _random_tier_case(seed, n_req=n_req, n_kv=n_kv, G=G, d=d, S=S,
                          steps=4, mem_kv=mem_kv, invalidate=inval)
    rng, page, NB, L, layer = c["rng"], c["page"], c["NB"], c["L"], c["layer"]
    MP = c["MP"]
    tier = T.Tier(num_layers=L, num_blocks=NB, n_kv=n_kv, page=page, d=d,
                  hot_slots=S, max_reqs=n_req, max_pages=MP, n_vslots=16,
                  offload_k=mem_kv, device=dev)
    r5, stg = tier.residency, tier.staging
    Vb = torch.from_numpy(c["V"]).to(torch.bfloat16)           # (NB,P,kv,d)
    Kb = torch.from_numpy(c["K"]).to(torch.bfloat16)
    # pinned pool holds every page; 12 blocks are staged and not flushed
    # (their pinned copy is garbage until the write-through)
    tier.pool.host[layer].copy_(Vb.permute(0, 2, 1, 3))
    if mem_kv:
        tier.pool_k.host[layer].copy_(Kb.permute(0, 2, 1, 3))
    r5.pool_valid.fill_(1)
    staged = rng.choice(NB, 12, replace=False)
    vbo = np.full(NB, -1, np.int32)
    for i, blk in enumerate(staged):
        vbo[blk] = i
        stg.v_pool[layer, i].copy_(Vb[blk])
        tier.pool.host[layer, blk].fill_(7.0)
        if mem_kv:
            stg.k_pool[layer, i].copy_(Kb[blk])
            tier.pool_k.host[layer, blk].fill_(-3.0)
        r5.pool_valid[layer, :, blk] = 0
    # two more blocks neither flushed nor staged: both sides read the pool
    for blk in rng.choice(np.setdiff1d(np.arange(NB), staged), 2,
                          replace=False):
        r5.pool_valid[layer, :, blk] = 0
    stg.vbo.copy_(torch.from_numpy(vbo))
    # oracle mirrors (int16 bits)
    o_pool = tier.pool.host.view(torch.int16).numpy().copy()
    o_poolk = tier.pool_k.host.view(torch.int16).numpy().copy() if mem_kv \
        else None
    o_valid = r5.pool_valid.cpu().numpy().copy()
    o_p2s = np.full((L, n_kv, NB), -1, np.int32)
    o_s2p = np.full((L, n_kv, S), -1, np.int32)
    o_lru = np.zeros((n_kv, S), np.int32)
    o_hot = np.zeros((n_kv, S, page, d), np.int16)
    o_hotk = np.zeros_like(o_hot)
    v_pool16 = stg.v_pool[layer].view(torch.int16).cpu().numpy()
    k_pool16 = stg.k_pool[layer].view(torch.int16).cpu().numpy() if mem_kv \
        else None
    kv_true = torch.stack([Kb, Vb], 1).contiguous().to(dev)
    kv_dev = kv_true if not mem_kv else torch.zeros_like(kv_true)
    bt = torch.from_numpy(c["bt"]).to(dev)
    sl = torch.from_numpy(c["ctx"]).to(dev)
    st = _state(dev, n_req=n_req, n_kv=n_kv, G=G, d=d, NB=NB, MP=MP)
    q_all = O.bf16_round(rng.standard_normal(
        (len(c["sels"]), n_req, n_kv * G, d)).astype(np.float32))
    clock = 1
    o_ovf = False
    for s, (tab, cnt) in enumerate(c["sels"]):
        if inval and s == 2:
            qsl = np.arange(n_req + 1, dtype=np.int32)          # one token each
            r5.invalidate_written(bt, sl, torch.from_numpy(qsl).to(dev))
            O.invalidate_written(c["bt"], c["ctx"], qsl, page=page,
                                 page2slot=o_p2s, slot2page=o_s2p,
                                 pool_valid=o_valid)
        st.page_table.copy_(torch.from_numpy(tab))
        st.page_cnt.copy_(torch.from_numpy(cnt))
        q = torch.from_numpy(q_all[s]).to(torch.bfloat16).to(dev)
        out = torch.zeros(q.shape, dtype=torch.bfloat16, device=dev)
        T.mem_dynamic_decode(q, kv_dev, bt, sl, st, out, tier, layer,
                             scale=d ** -0.5, fetch=fetch)
        res = torch.zeros_like(out)
        A.sparse_paged_decode_batched_cuda(q, kv_true, bt, sl, st, res,
                                           scale=d ** -0.5)
        # the same decode without the plan's entry slots (page2slot lookups)
        out2 = torch.zeros_like(out)
        T.mem_decode_ptrsel(q, kv_dev, bt, sl, st, out2, tier, layer,
                            scale=d ** -0.5)
        torch.cuda.synchronize()
        assert torch.equal(out, out2), s
        clock += 1
        fl, ovf = O.residency_step(tab, cnt, c["bt"], c["ctx"], page=page,
                                   page2slot=o_p2s[layer], slot2page=o_s2p[layer],
                                   lru=o_lru, clock=clock)
        o_ovf = o_ovf or ovf
        valid_k = o_valid[layer].copy()        # validity the fetch decides on
        O.residency_fetch(fl, hot=o_hot, pool=o_pool, pool_valid=o_valid[layer],
                          vbo=vbo, v_pool=v_pool16, layer=layer)
        if mem_kv:
            # K shares the list and the source decision made on V's validity
            for kvh, blk, slot in fl:
                if valid_k[kvh, blk] > 0 or vbo[blk] < 0:
                    o_hotk[kvh, slot] = o_poolk[layer, blk, kvh]
                else:
                    o_hotk[kvh, slot] = k_pool16[vbo[blk], :, kvh]
                    o_poolk[layer, blk, kvh] = k_pool16[vbo[blk], :, kvh]
        assert np.array_equal(r5.page2slot.cpu().numpy(), o_p2s), s
        assert np.array_equal(r5.slot2page.cpu().numpy(), o_s2p), s
        assert np.array_equal(r5.lru_clock[layer].cpu().numpy(), o_lru), s
        assert np.array_equal(r5.pool_valid.cpu().numpy(), o_valid), s
        assert int(r5.overflow[0]) == int(o_ovf), s
        got = set()
        fc = r5.fetch_cnt.cpu().numpy()
        fls = r5.fetch_list.cpu().numpy()
        for kvh in range(n_kv):
            for e in range(fc[kvh]):
                got.add((kvh, int(fls[kvh, e, 0]), int(fls[kvh, e, 1])))
        assert got == set(fl), s
        hot = _bits(r5.hot[layer])
        res_mask = o_s2p[layer] >= 0
        assert np.array_equal(hot[res_mask], o_hot[res_mask]), s
        if mem_kv:
            assert np.array_equal(_bits(r5.hot_k[layer])[res_mask],
                                  o_hotk[res_mask]), s
        assert np.array_equal(tier.pool.host.view(torch.int16).numpy(), o_pool)
        # the tier serves the true bytes: bitwise equal to the resident decode
        assert torch.equal(out, res), s
        ref = O.sparse_decode(q_all[s], c["K"], c["V"], c["bt"], c["ctx"], tab,
                              cnt, scale=d ** -0.5, G=G)
        np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=ATOL,
                                   rtol=RTOL)
    r5.assert_maps_inverse()
    if S == 6:
        assert int(r5.overflow[0]) == 1


def test_tier_plan_is_graph_capturable(dev):
    """plan + fetch + decode replay in a CUDA graph: the clock advances once
    per replay and the maps match eager calls on a twin tier."""
    c = _random_tier_case(7, n_req=3, n_kv=2, G=4, d=128, S=32, steps=1)
    NB, MP, page = c["NB"], c["MP"], c["page"]
    tiers = []
    for _ in range(2):
        t = T.Tier(num_layers=2, num_blocks=NB, n_kv=2, page=page, d=128,
                   hot_slots=32, max_reqs=3, max_pages=MP, n_vslots=4,
                   device=dev)
        Vb = torch.from_numpy(c["V"]).to(torch.bfloat16)
        t.pool.host[1].copy_(Vb.permute(0, 2, 1, 3))
        t.residency.pool_valid.fill_(1)
        tiers.append(t)
    Kb = torch.from_numpy(c["K"]).to(torch.bfloat16)
    Vb = torch.from_numpy(c["V"]).to(torch.bfloat16)
    kv = torch.stack([Kb, Vb], 1).contiguous().to(dev)
    bt = torch.from_numpy(c["bt"]).to(dev)
    sl = torch.from_numpy(c["ctx"]).to(dev)
    st = _state(dev, n_req=3, n_kv=2, G=4, d=128, NB=NB, MP=MP)
    tab, cnt = c["sels"][0]
    st.page_table.copy_(torch.from_numpy(tab))
    st.page_cnt.copy_(torch.from_numpy(cnt))
    q = torch.randn(3, 8, 128, device=dev).to(torch.bfloat16)
    outs = [torch.zeros_like(q) for _ in range(2)]
    T.mem_dynamic_decode(q, kv, bt, sl, st, outs[0], tiers[0], 1)   # warm
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
        T.mem_dynamic_decode(q, kv, bt, sl, st, outs[0], tiers[0], 1)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        g.replay()
    for _ in range(4):
        T.mem_dynamic_decode(q, kv, bt, sl, st, outs[1], tiers[1], 1)
    torch.cuda.synchronize()
    a, b = tiers[0].residency, tiers[1].residency
    assert int(a.clock[0]) == int(b.clock[0]) == 5
    assert int(a.clock[1]) == 0
    assert torch.equal(a.page2slot, b.page2slot)
    assert torch.equal(a.lru_clock, b.lru_clock)
    assert torch.equal(outs[0], outs[1])


def test_invalidate_golden(dev):
    z = load_golden("tier_invalidate")
    L, n_kv, NB = z["page2slot_init"].shape
    S = z["slot2page_init"].shape[2]
    r5 = T.Residency(num_layers=L, num_blocks=NB, n_kv=n_kv, hot_slots=S,
                     page=int(z["page"][0]), d=64, max_reqs=4, max_pages=8,
                     device=dev)
    r5.page2slot.copy_(torch.from_numpy(z["page2slot_init"]))
    r5.slot2page.copy_(torch.from_numpy(z["slot2page_init"]))
    r5.pool_valid.copy_(torch.from_numpy(z["pool_valid_init"]))
    r5.invalidate_written(torch.from_numpy(z["block_table"]).to(dev),
                          torch.from_numpy(z["seq_lens"]).to(dev),
                          torch.from_numpy(z["query_start_loc"]).to(dev))
    torch.cuda.synchronize()
    assert np.array_equal(r5.page2slot.cpu().numpy(), z["page2slot"])
    assert np.array_equal(r5.slot2page.cpu().numpy(), z["slot2page"])
    assert np.array_equal(r5.pool_valid.cpu().numpy(), z["pool_valid"])


@pytest.mark.parametrize("mem_kv", [False, True])
def test_tier_dma_coalesced_runs(mem_kv, dev):
    """A fresh hot buffer takes victims in slot order, so one request whose
    blocks are consecutive installs consecutive blocks into consecutive
    slots: the copy-engine plan coalesces them into a few strided 2-D runs
    (staged blocks break runs and go to the staged-only kernel), and the hot
    buffer, pool and validity end bit-equal to the kernel fetch's."""
    n_kv, G, d, page, S = 2, 4, 128, 16, 64
    NB, MP = 80, 48
    res = {}
    for mode in ("kernel", "dma"):
        tier = T.Tier(num_layers=1, num_blocks=NB, n_kv=n_kv, page=page, d=d,
                      hot_slots=S, max_reqs=1, max_pages=MP, n_vslots=8,
                      offload_k=mem_kv, device=dev)
        r5, stg = tier.residency, tier.staging
        g = torch.Generator().manual_seed(5)
        host = torch.randn(tier.pool.host.shape, generator=g)
        tier.pool.host.copy_(host.to(torch.bfloat16))
        if mem_kv:
            tier.pool_k.host.copy_((-host).to(torch.bfloat16))
        r5.pool_valid.fill_(1)
        for i, blk in enumerate((20, 31)):          # staged, not flushed
            stg.vbo[blk] = i
            stg.v_pool[0, i].fill_(float(i + 2))
            if mem_kv:
                stg.k_pool[0, i].fill_(float(-i - 2))
            r5.pool_valid[0, :, blk] = 0
        bt = torch.arange(10, 10 + MP, dtype=torch.int32,
                          device=dev)[None].contiguous()
        sl = torch.tensor([MP * page], dtype=torch.int32, device=dev)
        tab = torch.full((1, n_kv, MP), -1, dtype=torch.int32, device=dev)
        cnt = torch.tensor([[40, 33]], dtype=torch.int32, device=dev)
        tab[0, 0, :40] = torch.arange(40, dtype=torch.int32)
        tab[0, 1, :33] = torch.arange(5, 38, dtype=torch.int32)
        if mode == "kernel":
            tier.step(0, tab, cnt, bt, sl, 1)
        else:
            r5.gather_plan(0, tab, cnt, bt, sl, 1)
            runs, staged = r5.build_dma_plan(0, tier.pool.dev_view, 1,
                                             tier.pool_k.dev_view
                                             if mem_kv else None)
            assert staged
            assert 0 < len(runs) <= 6, len(runs)
            assert sum(r.height for r in runs) == 40 + 33 - 2 - 2
            ev = r5.gather_fetch_dma(0, stg, tier.pool.dev_view, 1,
                                     tier.copy_engine,
                                     poolk=tier.pool_k.dev_view
                                     if mem_kv else None)
            torch.cuda.current_stream(dev).wait_event(ev)
        torch.cuda.synchronize(dev)
        res[mode] = (_bits(r5.hot), _bits(r5.hot_k) if mem_kv else None,
                     tier.pool.host.view(torch.int16).numpy().copy(),
                     r5.pool_valid.cpu().numpy(),
                     r5.slot2page.cpu().numpy())
    for a, b in zip(res["kernel"], res["dma"]):
        if a is not None:
            assert np.array_equal(a, b)


def test_tier_plan_empty_batch(dev):
    """An empty batch is a valid plan call: status 0, no installs, the maps
    unchanged and the step clock advanced once (reference residency.py
    gather_plan increments the clock before its kernels)."""
    NB, MP = 64, 8
    t = T.Tier(num_layers=1, num_blocks=NB, n_kv=2, page=16, d=128,
               hot_slots=16, max_reqs=2, max_pages=MP, n_vslots=4, device=dev)
    r5 = t.residency
    tab = torch.full((2, 2, MP), -1, dtype=torch.int32, device=dev)
    cnt = torch.zeros((2, 2), dtype=torch.int32, device=dev)
    bt = torch.zeros((2, MP), dtype=torch.int32, device=dev)
    sl = torch.zeros((2,), dtype=torch.int32, device=dev)
    p2s, lru = r5.page2slot.clone(), r5.lru_clock.clone()
    c0 = int(r5.clock[0])
    r5.gather_plan(0, tab, cnt, bt, sl, 0)
    torch.cuda.synchronize()
    assert int(r5.clock[0]) == c0 + 1
    assert int(r5.fetch_cnt.sum()) == 0
    assert torch.equal(r5.page2slot, p2s)
    assert torch.equal(r5.lru_clock, lru)


@pytest.mark.parametrize("mem_kv", [False, True])
def test_install_decode_equals_plan_fetch_decode(mem_kv, dev):
    """The decode that fetches the plan's installs itself ends every step
    with the same output, hot buffer, pinned pool and validity as plan +
    separate fetch kernel + decode (staged unflushed pages included)."""
    c = _random_tier_case(9, n_req=5, n_kv=4, G=4, d=128, S=48, steps=5,
                          mem_kv=mem_kv)
    NB, MP, L, layer = c["NB"], c["MP"], c["L"], c["layer"]
    Vb = torch.from_numpy(c["V"]).to(torch.bfloat16)
    Kb = torch.from_numpy(c["K"]).to(torch.bfloat16)
    rng = np.random.default_rng(9)
    staged = rng.choice(NB, 10, replace=False)
    tiers = []
    for _ in range(2):
        t = T.Tier(num_layers=L, num_blocks=NB, n_kv=4, page=16, d=128,
                   hot_slots=48, max_reqs=5, max_pages=MP, n_vslots=16,
                   offload_k=mem_kv, device=dev)
        t.pool.host[layer].copy_(Vb.permute(0, 2, 1, 3))
        if mem_kv:
            t.pool_k.host[layer].copy_(Kb.permute(0, 2, 1, 3))
        t.residency.pool_valid.fill_(1)
        vbo = np.full(NB, -1, np.int32)
        for i, blk in enumerate(staged):
            vbo[blk] = i
            t.staging.v_pool[layer, i].copy_(Vb[blk])
            t.pool.host[layer, blk].fill_(5.0)
            if mem_kv:
                t.staging.k_pool[layer, i].copy_(Kb[blk])
                t.pool_k.host[layer, blk].fill_(-2.0)
            t.residency.pool_valid[layer, :, blk] = 0
        t.staging.vbo.copy_(torch.from_numpy(vbo))
        tiers.append(t)
    kv_true = torch.stack([Kb, Vb], 1).contiguous().to(dev)
    kv_dev = kv_true if not mem_kv else torch.zeros_like(kv_true)
    bt = torch.from_numpy(c["bt"]).to(dev)
    sl = torch.from_numpy(c["ctx"]).to(dev)
    st = _state(dev, n_req=5, n_kv=4, G=4, d=128, NB=NB, MP=MP)
    for s, (tab, cnt) in enumerate(c["sels"]):
        st.page_table.copy_(torch.from_numpy(tab))
        st.page_cnt.copy_(torch.from_numpy(cnt))
        q = torch.randn(5, 16, 128, device=dev).to(torch.bfloat16)
        outs = [torch.zeros_like(q) for _ in range(2)]
        # tier 0: the product path (plan, decode fetching the installs)
        T.mem_dynamic_decode(q, kv_dev, bt, sl, st, outs[0], tiers[0], layer,
                             scale=128 ** -0.5)
        # tier 1: plan + separate fetch kernel + decode
        r1 = tiers[1].residency
        tiers[1].step(layer, st.page_table, st.page_cnt, bt, sl, 5)
        T.mem_decode_ptrsel(q, kv_dev, bt, sl, st, outs[1], tiers[1], layer,
                            scale=128 ** -0.5, entry_slots=r1.miss_pages)
        torch.cuda.synchronize()
        a, b = tiers[0].residency, tiers[1].residency
        assert torch.equal(outs[0], outs[1]), s
        assert torch.equal(a.page2slot, b.page2slot), s
        assert torch.equal(a.pool_valid, b.pool_valid), s
        res_mask = a.slot2page[layer] >= 0
        assert torch.equal(a.hot[layer][res_mask], b.hot[layer][res_mask]), s
        if mem_kv:
            assert torch.equal(a.hot_k[layer][res_mask],
                               b.hot_k[layer][res_mask]), s
        assert torch.equal(tiers[0].pool.host, tiers[1].pool.host), s
        if mem_kv:
            assert torch.equal(tiers[0].pool_k.host, tiers[1].pool_k.host), s
