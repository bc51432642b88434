"""AmassConfig -- the reference's configuration object, same fields and rules.

Field names, defaults and validation follow the reference's
``src/amass/config.py:26-140`` so a config that loads there loads here; the
load path (``AMASS_CONFIG`` as a JSON/YAML file path or inline JSON, plus
explicit overrides, unknown keys rejected) follows ``config.py:142-165``.
``use_cuda`` is accepted for compatibility; this build has one path (the
sm_100a kernels) and no fallback, so the flag has no effect.
"""
from __future__ import annotations

import dataclasses
import json
import os
from typing import Literal, Optional

Variant = Literal["fast", "mem-v", "mem-kv"]


@dataclasses.dataclass(frozen=True)
class AmassConfig:
    variant: Variant = "mem-v"
    coverage: float = 0.95
    budget: Optional[float] = None
    table: str = "kv-union"
    sink_pages: int = 1
    window_pages: int = 1
    r8_screen: bool = False
    r8_rank: int = 8
    score: str = "clse"
    quad_rank: int = 2
    quad_v_bits: int = 4
    quad_combine: str = "nrm"
    quad_c_bits: int = 4
    quad_c_grain: str = "token"
    hot_slots: int = 2048
    v_blocks: Optional[int] = None
    max_pool_gb: float = 256.0
    use_cuda: bool = True
    force_eager: bool = False

    @property
    def is_mem(self) -> bool:
        return self.variant in ("mem-v", "mem-kv")

    @property
    def offload_k(self) -> bool:
        return self.variant == "mem-kv"

    def __post_init__(self) -> None:
        checks = [
            (self.variant in ("fast", "mem-v", "mem-kv"),
             f"unknown variant {self.variant!r}"),
            (0.0 < self.coverage <= 1.0,
             f"coverage must be in (0,1], got {self.coverage}"),
            (self.budget is None or 0.0 < self.budget <= 1.0,
             f"budget must be in (0,1], got {self.budget}"),
            (self.score in ("r8", "quad", "clse"),
             f"score must be 'r8', 'quad' or 'clse', got {self.score!r}"),
            (self.quad_rank >= 1, f"quad_rank must be >= 1, got "
             f"{self.quad_rank}"),
            (self.quad_v_bits in (4, 8),
             f"quad_v_bits must be 4 or 8, got {self.quad_v_bits}"),
            (self.quad_combine in ("max", "nrm"),
             f"quad_combine must be 'max' or 'nrm', got "
             f"{self.quad_combine!r}"),
            (self.quad_c_bits in (4, 8),
             f"quad_c_bits must be 4 or 8, got {self.quad_c_bits}"),
            (self.quad_c_grain in ("token", "page"),
             f"quad_c_grain must be 'token' or 'page', got "
             f"{self.quad_c_grain!r}"),
        ]
        for ok, msg in checks:
            if not ok:
                raise ValueError(msg)
        # mem-kv cannot scan a resident K, so it always uses the r8 screen
        if self.offload_k and not self.r8_screen:
            object.__setattr__(self, "r8_screen", True)

    @classmethod
    def load(cls, overrides: Optional[dict] = None) -> "AmassConfig":
        data: dict = {}
        spec = os.environ.get("AMASS_CONFIG")
        if spec:
            if os.path.isfile(spec):
                with open(spec) as fh:
                    text = fh.read()
                if spec.endswith((".yaml", ".yml")):
                    import yaml
                    data = yaml.safe_load(text) or {}
                else:
                    data = json.loads(text)
            else:
                data = json.loads(spec)
        if overrides:
            data.update({k: v for k, v in overrides.items() if v is not None})
        unknown = set(data) - {f.name for f in dataclasses.fields(cls)}
        if unknown:
            raise ValueError(f"unknown AmassConfig keys: {sorted(unknown)}")
        return cls(**data)
