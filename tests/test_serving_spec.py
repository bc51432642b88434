"""The K-only cache-spec patch (engine half of the mem tier's VRAM saving):
full-attention specs lose their V half, anything else is refused."""
import pytest
import torch

from amass_kv_b200.serving import patch_kv_cache_spec_k_only

spec_mod = pytest.importorskip("vllm.v1.kv_cache_interface")


def _layer_cls(spec):
    class FakeAttention:
        def get_kv_cache_spec(self, vllm_config=None):
            return spec
    return FakeAttention


def test_full_attention_becomes_k_only():
    spec = spec_mod.FullAttentionSpec(16, num_kv_heads=8, head_size=128,
                                      dtype=torch.bfloat16)
    cls = _layer_cls(spec)
    patch_kv_cache_spec_k_only(cls)
    patch_kv_cache_spec_k_only(cls)          # idempotent
    out = cls().get_kv_cache_spec(None)
    assert out.head_size_v == 0 and out.head_size == 128
    assert out.page_size_bytes * 2 == spec.page_size_bytes


def test_refuses_what_it_cannot_serve():
    sw = spec_mod.FullAttentionSpec(16, num_kv_heads=8, head_size=128,
                                    dtype=torch.bfloat16, sliding_window=512)
    cls = _layer_cls(sw)
    patch_kv_cache_spec_k_only(cls)
    with pytest.raises(RuntimeError):
        cls().get_kv_cache_spec(None)
    asym = spec_mod.FullAttentionSpec(16, num_kv_heads=8, head_size=128,
                                      dtype=torch.bfloat16, head_size_v=64)
    cls = _layer_cls(asym)
    patch_kv_cache_spec_k_only(cls)
    with pytest.raises(RuntimeError):
        cls().get_kv_cache_spec(None)
