"""Route the reference package ``avqa`` through this package's CUDA path.

``install()`` is the maintainer's patch that lets the reference's own
``avqa.AVQAttention`` run on the B200 library with ``backend.name = "cuda"``:

* ``Backend.create("cuda")`` (reference ``backend.py:48-102``) returns
  :class:`avqa_b200.backend.CUDABackend`; other names keep the reference's
  behaviour;
* ``BackendConfig.__post_init__`` (``config.py:191-195``) accepts ``"cuda"``;
* ``run_pipeline`` (``pipeline.py:276-399``) hands a module whose backend is
  a :class:`CUDABackend` to :func:`cuda_run_pipeline`.  The reference's
  ``attention_module`` imported the function by name
  (``from avqa.pipeline import run_pipeline``), so the hook is installed in
  both modules.

``install()`` returns a function that undoes the patch.  It needs the
reference package importable as ``avqa``.
"""
from __future__ import annotations

from typing import Callable


def install() -> Callable[[], None]:
    import avqa.attention_module as ref_module
    import avqa.backend as ref_backend
    import avqa.config as ref_config
    import avqa.pipeline as ref_pipeline

    from avqa_b200.attention_module import cuda_run_pipeline
    from avqa_b200.backend import CUDABackend

    saved = (ref_backend.Backend.__dict__["create"], ref_config.BackendConfig.__post_init__,
             ref_pipeline.run_pipeline, ref_module.run_pipeline)
    orig_create = saved[0].__func__
    orig_post_init = saved[1]
    orig_run = saved[2]

    def create(cls, name: str = "torch"):
        return CUDABackend() if name == "cuda" else orig_create(cls, name)

    def post_init(self) -> None:
        if self.name != "cuda":
            orig_post_init(self)

    def run_pipeline(state, query, key, value, mask, kv_cache):
        if isinstance(state.backend, CUDABackend):
            return cuda_run_pipeline(state, query, key, value, mask, kv_cache)
        return orig_run(state, query, key, value, mask, kv_cache)

    ref_backend.Backend.create = classmethod(create)
    ref_config.BackendConfig.__post_init__ = post_init
    ref_pipeline.run_pipeline = run_pipeline
    ref_module.run_pipeline = run_pipeline

    def uninstall() -> None:
        ref_backend.Backend.create = saved[0]
        ref_config.BackendConfig.__post_init__ = saved[1]
        ref_pipeline.run_pipeline = saved[2]
        ref_module.run_pipeline = saved[3]

    return uninstall


__all__ = ["install"]
