"""Loading of the golden fixtures recorded from the reference (tests/golden)."""
from __future__ import annotations

import hashlib
import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
TD = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def case_names() -> list[str]:
    return sorted(p.stem for p in GOLDEN.glob("*.npz"))


def from_bits(a: np.ndarray, dt: str) -> np.ndarray:
    """Stored array -> float32 values (bf16 is stored as uint16 bit patterns)."""
    if dt == "bf16" and a.dtype == np.uint16:
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a.astype(np.float32)


def to_torch(a: np.ndarray, dt: str) -> torch.Tensor:
    return torch.from_numpy(from_bits(a, dt).copy()).to(TD[dt])


@dataclass
class Golden:
    name: str
    meta: dict
    arrs: dict

    @property
    def w(self) -> dict:
        return self.meta["workload"]

    @property
    def dt(self) -> str:
        return self.w["dtype"]

    def get(self, key: str) -> np.ndarray:
        return self.arrs[key]

    def f(self, key: str) -> np.ndarray:
        return from_bits(self.arrs[key], self.dt)

    def mask_for(self, t_q: int, t_k: int):
        """The call's mask (True = attend): the recorded user mask, the causal
        mask of config.causal for a ``t_q`` x ``t_k`` call, or None."""
        kind = self.meta.get("mask")
        if kind == "causal":
            i = np.arange(t_q)[:, None]
            return np.arange(t_k)[None, :] <= i + (t_k - t_q)
        if kind in ("user2", "user4"):
            return self.arrs["mask"].astype(bool)
        return None

    def inputs(self):
        """fp32-valued numpy ``(q, k, v)`` in module layout ``[B, T/S, E]``."""
        if "q" in self.arrs:
            return self.f("q"), self.f("k"), self.f("v")
        w = self.w
        torch.manual_seed(w["seed"])
        E = w["H"] * w["D"]
        q = torch.randn(w["B"], w["T"], E)
        k = torch.randn(w["B"], w["S"], E)
        v = torch.randn(w["B"], w["S"], E)
        digest = hashlib.sha256(b"".join(t.numpy().tobytes() for t in (q, k, v))).hexdigest()
        assert digest == self.meta["qkv_sha256"], "regenerated README inputs differ from the recorded ones"
        return q.numpy(), k.numpy(), v.numpy()


def load(name: str) -> Golden:
    z = np.load(GOLDEN / f"{name}.npz")
    arrs = {k: z[k] for k in z.files}
    meta = json.loads(bytes(arrs.pop("meta_json")).decode())
    return Golden(name, meta, arrs)
