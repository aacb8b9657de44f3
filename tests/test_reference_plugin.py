"""The drop-in into the reference package itself (``avqa_b200.reference_plugin``).

Runs where the reference source is present (it does not travel with the
tests; skipped elsewhere).  With the patch installed, the reference's own
``avqa.AVQAttention`` built with ``backend.name = "cuda"`` must

* hold this package's ``CUDABackend`` (``Backend.create``);
* accept ``"cuda"`` in its ``BackendConfig``;
* send ``forward`` through ``cuda_run_pipeline``: with CPU tensors that
  function stops at its device check (the reference pipeline would return an
  output), after calling the reference module's own ``validate_inputs``;
* expose every attribute ``cuda_run_pipeline`` reads.

The torch backend's output is unchanged by the patch, and uninstalling
restores the reference exactly.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest
import torch

REF_SRC = Path(os.environ.get("AVQ_REFERENCE_SRC", "/root/reference/src"))
pytestmark = pytest.mark.skipif(not (REF_SRC / "avqa" / "__init__.py").exists(),
                                reason="reference source not present")


@pytest.fixture(scope="module")
def avqa():
    sys.path.insert(0, str(REF_SRC))
    try:
        import avqa as ref
        yield ref
    finally:
        sys.path.remove(str(REF_SRC))


def _config(ref, backend: str):
    from avqa.config import AttentionShapeConfig, BackendConfig, CodebookConfig, RoutingConfig
    return ref.AVQConfig(attention=AttentionShapeConfig(embed_dim=32, num_heads=2),
                         codebook=CodebookConfig(num_codewords=8, children_per_codeword=2),
                         routing=RoutingConfig(strategy="budget", refinement_budget=3),
                         backend=BackendConfig(name=backend))


def _torch_out(ref, seed: int = 0) -> torch.Tensor:
    torch.manual_seed(seed)
    m = ref.AVQAttention(_config(ref, "torch"), in_proj=False, out_proj=False)
    q, k, v = (torch.randn(1, 12, 32) for _ in range(3))
    return m(q, k, v)


def test_reference_module_routes_to_cuda_path(avqa) -> None:
    import avqa.attention_module as ref_module
    import avqa.pipeline as ref_pipeline
    from avqa.exceptions import ConfigurationError

    from avqa_b200 import reference_plugin
    from avqa_b200.backend import CUDABackend
    from avqa_b200.exceptions import DeviceError

    before = _torch_out(avqa)
    orig = (ref_pipeline.run_pipeline, ref_module.run_pipeline)
    with pytest.raises(ConfigurationError):
        _config(avqa, "cuda")
    uninstall = reference_plugin.install()
    try:
        m = avqa.AVQAttention(_config(avqa, "cuda"), in_proj=False, out_proj=False)
        assert isinstance(m.backend, CUDABackend)
        for attr in ("config", "codebook", "q_proj", "k_proj", "v_proj", "out_proj", "dropout", "validate_inputs",
                     "sync_codebook_device", "backend"):
            assert hasattr(m, attr), attr
        assert tuple(m.codebook.parents.shape) == (2, 8, 16) and tuple(m.codebook.children.shape) == (2, 8, 2, 16)
        q = torch.randn(1, 12, 32)
        with pytest.raises(DeviceError, match="cuda backend needs CUDA tensors"):
            m(q, q, q)
        # the reference's own input validation ran first (a rank-2 query is refused there)
        with pytest.raises(Exception) as info:
            m(q[0], q, q)
        assert not isinstance(info.value, DeviceError)
        assert torch.equal(_torch_out(avqa), before)
    finally:
        uninstall()
    assert (ref_pipeline.run_pipeline, ref_module.run_pipeline) == orig
    with pytest.raises(ConfigurationError):
        _config(avqa, "cuda")
    assert torch.equal(_torch_out(avqa), before)
