"""Generate the streaming-VQ fixtures in ``stream/`` by running the reference.

Run from the repository root in a container that has the reference source
(``python tests/golden/make_stream_golden.py [/path/to/reference]``; default
path ``/root/reference``).  Each case feeds a seeded sequence of key batches
through the reference's own ``avqa.streaming_vq.StreamingVQBuffer`` (CPU) and
records, per call, the keys and the returned ``[B, H]`` assignments, and at
the end the buffer's counts, aggregates and ``realize()`` output.  Tensors in
bf16 are stored as uint16 bit patterns, fp16 as float16.  The reference is
not needed at test time.

Cases cover one key per call (the token stream), batches with several heads
(the reference's head pairing ``i // B`` / key ``i // H`` for the flat rows),
many keys of one call landing on the same codeword (the fp32-accumulate,
narrow-once rounding of ``index_add_``), a zero-key call, a NaN key and fp16
distances that overflow.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
OUT = HERE / "stream"
TD = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}

# name: (dtype, H, M0, C, D, key batch sizes, key kind, seed)
CASES: dict[str, tuple] = {
    "h1_b8_f32": ("f32", 1, 4, 2, 8, [8, 8, 8], "normal", 0),
    "h4_mixed_bf16": ("bf16", 4, 16, 4, 64, [3, 1, 5, 0, 2, 7], "normal", 1),
    "h2_tokens_f16": ("f16", 2, 32, 4, 128, [1] * 24, "normal", 2),
    "h3_collide_bf16": ("bf16", 3, 4, 2, 32, [16, 16], "spread", 3),
    "h3_collide_f32": ("f32", 3, 4, 2, 32, [16, 16], "spread", 4),
    "h2_nan_f16": ("f16", 2, 8, 2, 16, [4, 3], "nan", 5),
    "h2_big_f16": ("f16", 2, 8, 2, 16, [5], "big", 6),
    "h5_b9_bf16": ("bf16", 5, 12, 3, 48, [9, 4], "normal", 7),
}


def bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.detach().cpu().numpy()


def make_keys(kind: str, B: int, D: int, g: torch.Generator) -> torch.Tensor:
    x = torch.randn(B, D, generator=g)
    if kind == "spread":
        # widely spread magnitudes per key: in bf16 the running sums of one
        # codeword round differently when accumulated in fp32 once vs per row
        x = x * torch.exp2(torch.randint(-6, 7, (B, 1), generator=g).float())
    elif kind == "nan" and B > 1:
        x[1, 3] = float("nan")
    elif kind == "big":
        x = x * 300.0  # fp16: k_sq and the cross terms overflow to inf
    return x


def run_case(name: str, spec: tuple, ref_root: Path) -> dict:
    sys.path.insert(0, str(ref_root / "src"))
    from avqa.streaming_vq import StreamingVQBuffer
    dt, H, M0, C, D, batches, kind, seed = spec
    g = torch.Generator().manual_seed(seed)
    parents = (torch.randn(H, M0, D, generator=g)).to(TD[dt])
    children = (parents.float()[:, :, None] + 0.3 * torch.randn(H, M0, C, D, generator=g)).to(TD[dt])
    if kind == "big":
        parents, children = (parents.float() * 300).to(TD[dt]), (children.float() * 300).to(TD[dt])
    buf = StreamingVQBuffer(num_heads=H, num_parents=M0, children_per_parent=C, head_dim=D, dtype=TD[dt])
    arrs = {"parents": bits(parents), "children": bits(children)}
    for i, B in enumerate(batches):
        keys = make_keys(kind, B, D, g).to(TD[dt])
        p, c = buf.extend(keys, parents, children)
        arrs[f"keys{i}"] = bits(keys)
        arrs[f"passign{i}"], arrs[f"cassign{i}"] = p.numpy(), c.numpy()
    arrs["pcnt"], arrs["ccnt"] = buf.parent_counts.numpy(), buf.child_counts.numpy()
    arrs["pagg"], arrs["cagg"] = bits(buf.parent_aggregates), bits(buf.child_aggregates)
    r = buf.realize()
    arrs["rec_passign"], arrs["rec_cassign"] = r.parent_assignments.numpy(), r.child_assignments.numpy()
    arrs["real_pcnt"], arrs["real_ccnt"] = bits(r.parent_counts), bits(r.child_counts)
    meta = dict(dtype=dt, H=H, M0=M0, C=C, D=D, batches=batches, kind=kind, seed=seed, size=len(buf))
    arrs["meta_json"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    return arrs


def main() -> None:
    ref_root = Path(sys.argv[1]) if len(sys.argv) > 1 else Path("/root/reference")
    torch.set_num_threads(1)
    OUT.mkdir(exist_ok=True)
    for name, spec in CASES.items():
        arrs = run_case(name, spec, ref_root)
        np.savez_compressed(OUT / f"{name}.npz", **arrs)
        print(name, "saved", sum(a.nbytes for a in arrs.values()), "bytes")


if __name__ == "__main__":
    main()
