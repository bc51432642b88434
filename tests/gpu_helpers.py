"""Helpers shared by the GPU parity tests: load a golden/synthetic case onto
the device in the reference layouts."""
import numpy as np
import torch

from amass_kv_b200.attention import ensure_stage_b_buffers
from amass_kv_b200.selection import QuadState
from tests.conftest import bits_to_f32


def to_dev_bf16_bits(bits, dev):
    return torch.from_numpy(np.ascontiguousarray(bits)).view(
        torch.bfloat16).to(dev)


def f32_to_bf16_dev(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(dev).to(
        torch.bfloat16)


class DevCase:
    """A quad case resident on `dev`: q, kv_cache, block_table, seq_lens and a
    filled QuadState (layer 0)."""

    def __init__(self, dev, *, q_bits=None, kv_bits=None, q=None, K=None,
                 V=None, block_table, seq_lens, mu, mu_s, Vq, V_s, sig2, G, r,
                 v_bits, page, MP, scale, budget=0.1, combine="nrm",
                 coverage=None, split=128):
        self.dev = dev
        if q_bits is not None:
            self.q = to_dev_bf16_bits(q_bits, dev)
            self.kv = to_dev_bf16_bits(kv_bits, dev)
        else:
            self.q = f32_to_bf16_dev(q, dev)
            self.kv = torch.stack([f32_to_bf16_dev(K, dev),
                                   f32_to_bf16_dev(V, dev)], dim=1).contiguous()
        self.bt = torch.from_numpy(np.ascontiguousarray(block_table)).to(dev)
        self.sl = torch.from_numpy(np.ascontiguousarray(seq_lens)).to(dev)
        self.n_req = int(block_table.shape[0])
        NB, _, page_, n_kv, d = self.kv.shape
        self.scale = float(scale)
        st = QuadState(dev, num_layers=1, num_blocks=NB, n_kv=n_kv, G=G,
                       head_dim=d, page=page, max_reqs=self.n_req,
                       max_pages=MP, rank=r, budget=budget, v_bits=v_bits,
                       combine=combine, coverage=coverage)
        st.quad_mu[0].copy_(torch.from_numpy(mu))
        st.mu_scale[0].copy_(torch.from_numpy(mu_s))
        st.quad_V[0].copy_(torch.from_numpy(Vq))
        st.V_scale[0].copy_(torch.from_numpy(V_s))
        st.quad_sig2[0].copy_(torch.from_numpy(sig2))
        st.score.fill_(float("nan"))
        if st.score_h is not None:
            st.score_h.fill_(float("nan"))
        ensure_stage_b_buffers(st, dev, split)
        self.st = st
        self.out = torch.zeros(self.q.shape, dtype=torch.bfloat16, device=dev)

    @classmethod
    def from_golden(cls, z, dev, **kw):
        G, r, vb, page, MP = [int(x) for x in z["meta"]]
        args = dict(q_bits=z["q"], kv_bits=z["kv"],
                    block_table=z["block_table"], seq_lens=z["seq_lens"],
                    mu=z["mu"], mu_s=z["mu_s"], Vq=z["Vq"], V_s=z["V_s"],
                    sig2=z["sig2"], G=G, r=r, v_bits=vb, page=page, MP=MP,
                    scale=float(z["scale"][0]), budget=float(z["budget"][0]),
                    combine=str(z["combine"][0]))
        args.update(kw)
        return cls(dev, **args)

    @classmethod
    def from_case(cls, c, dev, **kw):
        return cls(dev, q=c.q, K=c.K, V=c.V, block_table=c.block_table,
                   seq_lens=c.seq_lens, mu=c.mu, mu_s=c.mu_s, Vq=c.Vq,
                   V_s=c.V_s, sig2=c.sig2, G=c.G, r=c.r, v_bits=c.v_bits,
                   page=c.page, MP=c.MP, scale=c.scale, **kw)

    def host(self):
        """float32 numpy views for the oracle."""
        kv = self.kv.float().cpu().numpy()
        return dict(q=self.q.float().cpu().numpy(), K=kv[:, 0], V=kv[:, 1])
