"""Generate the golden fixtures in this folder by running the reference itself.

Run from the repository root in a container that has the reference source
(``python tests/golden/make_golden.py [/path/to/reference]``; default path
``/root/reference``).  For every case it builds seeded inputs, builds the
key-initialised codebook with the reference's own ``HierarchicalCodebook``
and ``EuclideanHierarchicalQuantizer``, runs the reference
``AVQAttention.forward`` (``TorchBackend``, CPU) and records the stage
outputs through wrappers around the reference's own functions:

* ``Backend.quantize``          -> assignments, aggregates, counts
* ``pipeline.online_softmax``   -> running max / denominator / numerator, probs
* ``compute_importance``        -> importance per routing call
* ``Router.select``             -> selected indices per routing call
* ``pipeline.per_query_beta``   -> HVAQ temperatures
* the module output

Fixtures are ``<case>.npz`` (numpy, compressed).  Tensors in bf16 are stored
as their uint16 bit patterns.  The reference is not needed at test time.
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from avqa_b200.workloads import Workload, make_decode_tokens, make_inputs  # noqa: E402

TD = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}

CASES: dict[str, dict] = {
    "c1_readme_f32": dict(w=Workload("c1", B=2, T=64, S=128, H=8, D=64, M0=64, C=4, P=8, dtype="f32",
                                     keys="readme", seed=0), strategy="budget"),
    "mix_bf16": dict(w=Workload("mix", B=2, T=256, S=256, H=2, D=128, M0=32, C=4, P=8, dtype="bf16",
                                keys="mixture", seed=1)),
    "mix_f32": dict(w=Workload("mix", B=2, T=128, S=128, H=2, D=128, M0=32, C=4, P=8, dtype="f32",
                               keys="mixture", seed=1)),
    "mix_f16": dict(w=Workload("mix", B=2, T=192, S=320, H=2, D=64, M0=24, C=4, P=6, dtype="f16",
                               keys="mixture", seed=11)),
    "mp_hvaq_f16": dict(w=Workload("mp", B=2, T=256, S=256, H=2, D=64, M0=32, C=4, P=12, dtype="f16",
                                   keys="student_t", seed=3, passes=3, pass_decay=0.5, hvaq=True)),
    "hvaq_lin_bf16": dict(w=Workload("hl", B=1, T=128, S=256, H=2, D=64, M0=32, C=4, P=8, dtype="bf16",
                                     keys="mixture", seed=5, hvaq=True), adaptive="linear", alpha=0.7),
    "mp_bf16": dict(w=Workload("mpb", B=1, T=128, S=256, H=2, D=64, M0=32, C=4, P=8, dtype="bf16",
                               keys="mixture", seed=6, passes=4, pass_decay=0.5)),
    "decode_bf16": dict(w=Workload("dec", B=2, T=1, S=128, H=2, D=64, M0=16, C=4, P=4, dtype="bf16",
                                   keys="aniso", seed=2, decode_steps=3, page_size=32)),
    "rope_bf16": dict(w=Workload("rope", B=1, T=64, S=512, H=2, D=64, M0=32, C=8, P=8, dtype="bf16",
                                 keys="mixture_rope", seed=4, q_chunk=32)),
    "mp_quirk_f32": dict(w=Workload("mpq", B=1, T=8, S=32, H=2, D=16, M0=4, C=2, P=4, dtype="f32",
                                    keys="mixture", seed=7, passes=2, pass_decay=1.0)),
    "single_key_bf16": dict(w=Workload("one", B=1, T=1, S=1, H=2, D=16, M0=8, C=2, P=4, dtype="bf16",
                                       keys="mixture", seed=8)),
    "empty_keys_bf16": dict(w=Workload("empty", B=1, T=3, S=0, H=2, D=16, M0=8, C=2, P=4, dtype="bf16",
                                       keys="mixture", seed=9)),
    "ties_bf16": dict(w=Workload("ties", B=1, T=4, S=16, H=1, D=8, M0=4, C=2, P=4, dtype="bf16",
                                 keys="mixture", seed=10), ties=True),
    # masks (pipeline.py:82-106): the causal mask of config.causal, a rank-2
    # user mask with one fully masked query, a rank-4 user mask, and the causal
    # mask with multi-pass refinement + HVAQ and with query chunks
    "causal_bf16": dict(w=Workload("causal", B=2, T=96, S=96, H=2, D=64, M0=16, C=4, P=6, dtype="bf16",
                                   keys="mixture", seed=12), mask="causal"),
    "mask2_f32": dict(w=Workload("mask2", B=1, T=40, S=64, H=2, D=32, M0=12, C=2, P=4, dtype="f32",
                                 keys="mixture", seed=13), mask="user2"),
    "mask4_bf16": dict(w=Workload("mask4", B=2, T=32, S=80, H=2, D=64, M0=16, C=4, P=5, dtype="bf16",
                                  keys="mixture", seed=14), mask="user4"),
    "causal_mp_hvaq_f16": dict(w=Workload("cmh", B=1, T=128, S=128, H=2, D=64, M0=24, C=4, P=8, dtype="f16",
                                          keys="student_t", seed=15, passes=2, pass_decay=0.5, hvaq=True),
                               mask="causal"),
    "causal_chunks_bf16": dict(w=Workload("cch", B=1, T=64, S=64, H=2, D=64, M0=16, C=4, P=6, dtype="bf16",
                                          keys="mixture", seed=16, q_chunk=32), mask="causal"),
    # BCAR online codebook adaptation (online_adaptation.py:37-127), two calls
    # in a row so that the second quantizes against the adapted codebook; B > 1
    # exercises the reference's tiling of the codebook over the batch
    "bcar_bf16": dict(w=Workload("bcar", B=1, T=64, S=200, H=2, D=64, M0=16, C=4, P=6, dtype="bf16",
                                 keys="mixture", seed=17), bcar=0.9, calls=2),
    "bcar_b2_f32": dict(w=Workload("bcar2", B=2, T=32, S=96, H=3, D=32, M0=12, C=2, P=4, dtype="f32",
                                   keys="mixture", seed=18), bcar=0.8, calls=2),
    "bcar_b3_f16": dict(w=Workload("bcar3", B=3, T=40, S=120, H=2, D=64, M0=16, C=4, P=5, dtype="f16",
                                   keys="aniso", seed=19), bcar=0.95, calls=2),
    # the dense path (backend.py:190-203): execution.mode = "reference" with the
    # causal mask, and refinement disabled with a rank-2 user mask
    "dense_ref_bf16": dict(w=Workload("dense", B=2, T=48, S=80, H=2, D=64, M0=16, C=4, P=6, dtype="bf16",
                                      keys="mixture", seed=20), mode="reference", mask="causal"),
    "dense_norefine_f32": dict(w=Workload("dense2", B=1, T=40, S=64, H=2, D=32, M0=12, C=2, P=4, dtype="f32",
                                          keys="mixture", seed=21), refine=False, mask="user2"),
}


def user_mask(w: Workload, rank: int) -> torch.Tensor:
    """A seeded boolean mask (True = attend, density 0.3); rank 2 ``[T, S]``
    with query 0 fully masked, or rank 4 ``[B, H, T, S]``."""
    g = torch.Generator().manual_seed(w.seed + 99)
    if rank == 2:
        m = torch.rand(w.T, w.S, generator=g) < 0.3
        m[0] = False
        return m
    return torch.rand(w.B, w.H, w.T, w.S, generator=g) < 0.3


def bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.detach().cpu().numpy()


def build_codebook(avqa, k_heads_b0: torch.Tensor, M0: int, C: int, seed: int):
    """The key-based recipe, with the reference's own classes (fp32)."""
    from avqa.codebook import HierarchicalCodebook
    from avqa.quantizer import EuclideanHierarchicalQuantizer
    H, S, D = k_heads_b0.shape
    k32 = k_heads_b0.float()
    cb = HierarchicalCodebook(num_heads=H, num_parents=M0, children_per_parent=C, head_dim=D)
    if S == 0:
        cb.initialize_parents_random(generator=torch.Generator().manual_seed(seed))
        return cb.parents.clone(), cb.children.clone()
    pos = torch.floor(torch.linspace(0, S - 1, M0, dtype=torch.float64)).long()
    cb.parents = k32[:, pos].clone()
    cb.initialize_children_around_parents(generator=torch.Generator().manual_seed(seed))
    r = EuclideanHierarchicalQuantizer().precompute(k32[None], k32[None], cb)
    cnt = r.child_counts[0]
    cb.children = torch.where((cnt > 0)[..., None], r.child_aggregates[0] / cnt.clamp_min(1.0)[..., None],
                              cb.children)
    cb.reproject_parents()
    return cb.parents.clone(), cb.children.clone()


def run_case(name: str, spec: dict, ref_root: Path) -> dict:
    sys.path.insert(0, str(ref_root / "src"))
    import avqa
    import avqa.multipass as amp
    import avqa.pipeline as apl
    import avqa.routing as art
    from avqa import AVQAttention
    from avqa.cache import InMemoryKVCache
    from avqa.config import (AttentionShapeConfig, AVQConfig, BackendConfig, CodebookConfig, HopfieldConfig,
                             RefinementConfig, RoutingConfig)

    w: Workload = spec["w"]
    dt = TD[w.dtype]
    q32, k32, v32 = make_inputs(w)
    if spec.get("ties"):
        # exact-tie stress: keys repeat a few rows, queries are identical rows
        k32 = k32[:, :4].repeat(1, w.S // 4, 1)
        q32 = q32[:, :1].repeat(1, w.T, 1)
    q, k, v = q32.to(dt), k32.to(dt), v32.to(dt)
    H, D = w.H, w.D
    kh = k.view(w.B, w.S, H, D).transpose(1, 2)
    parents, children = build_codebook(avqa, kh[0], w.M0, w.C, w.seed)
    if spec.get("ties"):
        children = children.clone()
        children[:, 1] = children[:, 0]  # duplicated parent -> exact distance ties
        parents = children.mean(2)

    mask = None
    if spec.get("mask") in ("user2", "user4"):
        mask = user_mask(w, 2 if spec["mask"] == "user2" else 4)
    from avqa.config import ExecutionConfig
    cfg = AVQConfig(
        causal=spec.get("mask") == "causal",
        execution=ExecutionConfig(mode=spec.get("mode", "optimized")),
        attention=AttentionShapeConfig(embed_dim=w.E, num_heads=H),
        codebook=CodebookConfig(num_codewords=w.M0, children_per_codeword=w.C,
                                bcar_enabled="bcar" in spec, bcar_decay=spec.get("bcar", 0.99)),
        routing=RoutingConfig(strategy=spec.get("strategy", "topp"), refinement_budget=w.P),
        refinement=RefinementConfig(enabled=spec.get("refine", True), passes=w.passes, pass_decay=w.pass_decay),
        backend=BackendConfig(hopfield=w.hvaq),
        hopfield=HopfieldConfig(adaptive=spec.get("adaptive", "entropy") if w.hvaq else "none",
                                alpha=spec.get("alpha", 1.0)),
    )
    mod = AVQAttention(cfg, in_proj=False, out_proj=False).eval()
    mod.codebook.parents = parents.clone()
    mod.codebook.children = children.clone()

    rec: dict[str, list] = {"quant": [], "softmax": [], "importance": [], "selected": [], "beta": [], "out": []}
    orig_q = mod.backend.quantize

    def q_wrap(*a, **kw):
        r = orig_q(*a, **kw)
        rec["quant"].append(r)
        return r
    mod.backend.quantize = q_wrap

    orig_os = apl.online_softmax

    def os_wrap(*a, **kw):
        st, pr = orig_os(*a, **kw)
        rec["softmax"].append((st.running_max[..., 0].clone(), st.running_denominator[..., 0].clone(),
                               st.running_numerator[..., 0, :].clone(), pr.clone()))
        return st, pr
    apl.online_softmax = os_wrap
    orig_ci_p, orig_ci_m = apl.compute_importance, amp.compute_importance

    def ci_wrap_p(*a, **kw):
        r = orig_ci_p(*a, **kw)
        rec["importance"].append(r.clone())
        return r

    def ci_wrap_m(*a, **kw):
        r = orig_ci_m(*a, **kw)
        rec["importance"].append(r.clone())
        return r
    apl.compute_importance, amp.compute_importance = ci_wrap_p, ci_wrap_m
    orig_sel = {cls: cls.select for cls in (art.TopPRouter, art.BudgetRouter)}

    def make_sel(cls):
        def sel_wrap(self, importance, budget):
            d = orig_sel[cls](self, importance, budget)
            rec["selected"].append(d.selected_indices.clone())
            return d
        return sel_wrap
    for cls in orig_sel:
        cls.select = make_sel(cls)
    orig_beta = apl.per_query_beta

    def beta_wrap(*a, **kw):
        r = orig_beta(*a, **kw)
        rec["beta"].append(r.clone())
        return r
    apl.per_query_beta = beta_wrap

    steps_meta = []
    try:
        with torch.no_grad():
            if w.decode_steps:
                cache = InMemoryKVCache(num_heads=H, head_dim_k=D, head_dim_v=D, dtype=dt)
                cache.append(kh, v.view(w.B, w.S, H, D).transpose(1, 2))
                toks = make_decode_tokens(w, w.decode_steps)
                for (qt, kt, vt) in toks:
                    rec["out"].append(mod(qt.to(dt), kt.to(dt), vt.to(dt), kv_cache=cache))
                    steps_meta.append(len(rec["selected"]))
            elif w.q_chunk:
                for c0 in range(0, w.T, w.q_chunk):
                    rec["out"].append(mod(q[:, c0:c0 + w.q_chunk], k, v))
            else:
                for _ in range(spec.get("calls", 1)):
                    rec["out"].append(mod(q, k, v, mask=mask))
                    rec.setdefault("cb", []).append((mod.codebook.parents.clone(), mod.codebook.children.clone()))
    finally:
        apl.online_softmax = orig_os
        apl.compute_importance, amp.compute_importance = orig_ci_p, orig_ci_m
        for cls, f in orig_sel.items():
            cls.select = f
        apl.per_query_beta = orig_beta

    meta = dict(name=name, workload=w.__dict__, config=cfg.to_dict(), ties=bool(spec.get("ties")),
                n_calls=len(rec["out"]), n_select=len(rec["selected"]), n_softmax=len(rec["softmax"]),
                n_importance=len(rec["importance"]), n_beta=len(rec["beta"]))
    arrs: dict[str, np.ndarray] = {"parents32": parents.numpy(), "children32": children.numpy()}
    meta["mask"] = spec.get("mask")
    if mask is not None:
        arrs["mask"] = mask.numpy().astype(np.uint8)
    if w.keys == "readme":
        # regenerated at test time from torch.manual_seed; the digest pins them
        meta["qkv_sha256"] = hashlib.sha256(b"".join(t.numpy().tobytes() for t in (q, k, v))).hexdigest()
    else:
        arrs.update(q=bits(q), k=bits(k), v=bits(v))
    for i, r in enumerate(rec["quant"]):
        arrs[f"quant{i}_passign"] = r.parent_assignments.numpy().astype(np.int32)
        arrs[f"quant{i}_cassign"] = r.child_assignments.numpy().astype(np.int32)
        arrs[f"quant{i}_pagg"] = bits(r.parent_aggregates)
        arrs[f"quant{i}_cagg"] = bits(r.child_aggregates)
        arrs[f"quant{i}_pcnt"] = r.parent_counts.float().numpy()
        arrs[f"quant{i}_ccnt"] = r.child_counts.float().numpy()
    for i, (m, l, a, p) in enumerate(rec["softmax"]):
        arrs[f"sm{i}_m"], arrs[f"sm{i}_l"], arrs[f"sm{i}_a"] = m.numpy(), l.numpy(), a.numpy()
        arrs[f"sm{i}_probs"] = bits(p)
    for i, t in enumerate(rec["importance"]):
        arrs[f"imp{i}"] = bits(t)
    for i, t in enumerate(rec["selected"]):
        arrs[f"sel{i}"] = t.numpy().astype(np.int32)
    for i, t in enumerate(rec["beta"]):
        arrs[f"beta{i}"] = bits(t)
    for i, (pp, cc) in enumerate(rec.get("cb", []) if "bcar" in spec else []):
        arrs[f"cb{i}_parents"], arrs[f"cb{i}_children"] = bits(pp), bits(cc)
    meta["bcar_decay"] = spec.get("bcar")
    meta["dense"] = spec.get("mode") == "reference" or spec.get("refine", True) is False
    for i, t in enumerate(rec["out"]):
        arrs[f"out{i}"] = t.float().numpy()
        meta[f"out{i}_dtype"] = str(t.dtype)
    if w.decode_steps:
        meta["decode_select_marks"] = steps_meta
    arrs["meta_json"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    return arrs


def main() -> None:
    ref_root = Path(sys.argv[1]) if len(sys.argv) > 1 else Path("/root/reference")
    only = set(sys.argv[2:])  # optional case names: regenerate just those
    torch.set_num_threads(1)
    for name, spec in CASES.items():
        if only and name not in only:
            continue
        arrs = run_case(name, spec, ref_root)
        np.savez_compressed(HERE / f"{name}.npz", **arrs)
        print(name, "saved", sum(a.nbytes for a in arrs.values()), "bytes")


if __name__ == "__main__":
    main()
