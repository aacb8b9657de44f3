"""Frozen configuration dataclasses of the AVQ-attention API.

Field names, defaults, validation rules and the JSON schema follow the
reference (``src/avqa/config.py:57-541``) so that configs serialised by one
load in the other.  The one deliberate difference: ``BackendConfig.name``
also admits ``"cuda"`` (the B200 backend); the reference admits only
``"torch"`` (``config.py:191-195``).
"""
from __future__ import annotations

import dataclasses
import json
from dataclasses import asdict, dataclass, field, fields
from pathlib import Path

from avqa_b200.exceptions import ConfigurationError

SCHEMA_VERSION: str = "1"
DEFAULT_EMA_DECAY: float = 0.99
BACKEND_NAMES = frozenset({"torch", "cuda"})


def require_positive(value: float, field_name: str) -> None:
    if value <= 0:
        raise ConfigurationError(f"{field_name} must be > 0, got {value}", {field_name: value})


def require_non_negative(value: float, field_name: str) -> None:
    if value < 0:
        raise ConfigurationError(f"{field_name} must be >= 0, got {value}", {field_name: value})


def require_in_range(value: float, lo: float, hi: float, field_name: str) -> None:
    if not lo <= value <= hi:
        raise ConfigurationError(f"{field_name} must be in [{lo}, {hi}], got {value}", {field_name: value})


def _require_choice(value: str, allowed: set[str] | frozenset[str], field_name: str) -> None:
    if value not in allowed:
        raise ConfigurationError(f"{field_name} must be one of {sorted(allowed)}, got {value!r}",
                                 {field_name: value})


@dataclass(frozen=True, slots=True)
class CodebookConfig:
    """Parents ``M0`` (``num_codewords``) and children per parent ``C``."""

    num_codewords: int = 64
    children_per_codeword: int = 4
    perturbation_scale: float = 0.1
    ema_decay: float = DEFAULT_EMA_DECAY
    commitment_loss_weight: float = 0.25
    max_depth: int = 2
    bcar_enabled: bool = False
    bcar_decay: float = 0.99

    def __post_init__(self) -> None:
        require_positive(self.num_codewords, "num_codewords")
        require_positive(self.children_per_codeword, "children_per_codeword")
        require_positive(self.perturbation_scale, "perturbation_scale")
        require_in_range(self.ema_decay, 0.0, 1.0, "ema_decay")
        require_non_negative(self.commitment_loss_weight, "commitment_loss_weight")
        require_in_range(self.bcar_decay, 0.0, 1.0, "bcar_decay")
        if self.max_depth != 2:
            raise ConfigurationError(f"max_depth={self.max_depth} is not supported; only max_depth=2",
                                     {"max_depth": self.max_depth})


@dataclass(frozen=True, slots=True)
class RoutingConfig:
    """Router strategy and the refinement budget ``P``."""

    strategy: str = "topp"
    refinement_budget: int = 8
    importance_temperature: float = 1.0

    def __post_init__(self) -> None:
        require_positive(self.refinement_budget, "refinement_budget")
        require_positive(self.importance_temperature, "importance_temperature")
        _require_choice(self.strategy, {"topp", "threshold", "budget"}, "routing.strategy")


@dataclass(frozen=True, slots=True)
class RefinementConfig:
    enabled: bool = True
    threshold: float = 0.0
    adaptive_budget: bool = False
    passes: int = 1
    pass_decay: float = 1.0

    def __post_init__(self) -> None:
        require_in_range(self.threshold, 0.0, 1.0, "threshold")


@dataclass(frozen=True, slots=True)
class MergeConfig:
    strategy: str = "probability"

    def __post_init__(self) -> None:
        _require_choice(self.strategy, {"probability", "weighted", "logit", "normalized"}, "merge.strategy")


@dataclass(frozen=True, slots=True)
class BackendConfig:
    """Backend selection.  This package implements ``"cuda"`` (the default
    here); ``"torch"`` is accepted so that the reference's JSON configs load,
    but constructing a module with it raises :class:`BackendError`."""

    name: str = "cuda"
    enable_autotune: bool = False
    skip_validation: bool = False
    hopfield: bool = False

    def __post_init__(self) -> None:
        _require_choice(self.name, BACKEND_NAMES, "backend.name")


@dataclass(frozen=True, slots=True)
class CacheConfig:
    enabled: bool = True
    max_size: int = 0

    def __post_init__(self) -> None:
        require_non_negative(self.max_size, "cache.max_size")


@dataclass(frozen=True, slots=True)
class PrecisionConfig:
    dtype: str = "float32"
    autocast: bool = False

    def __post_init__(self) -> None:
        _require_choice(self.dtype, {"float32", "float16", "bfloat16"}, "precision.dtype")


@dataclass(frozen=True, slots=True)
class ExecutionConfig:
    mode: str = "optimized"
    deterministic: bool = False
    seed: int = 0
    compile_enabled: bool = False
    causal_incremental: bool = False

    def __post_init__(self) -> None:
        _require_choice(self.mode, {"reference", "optimized", "research"}, "execution.mode")
        require_non_negative(self.seed, "execution.seed")


@dataclass(frozen=True, slots=True)
class HopfieldConfig:
    """HVAQ temperature schedule: ``adaptive`` in none/entropy/linear."""

    enabled: bool = False
    beta_init: float = 0.0
    adaptive: str = "none"
    alpha: float = 1.0
    learnable_parent_beta: bool = False
    learnable_alpha: bool = False

    def __post_init__(self) -> None:
        if self.beta_init < 0.0:
            raise ConfigurationError(f"hopfield.beta_init must be >= 0, got {self.beta_init}",
                                     {"hopfield.beta_init": self.beta_init})
        if self.alpha < 0.0:
            raise ConfigurationError(f"hopfield.alpha must be >= 0, got {self.alpha}", {"hopfield.alpha": self.alpha})


@dataclass(frozen=True, slots=True)
class AttentionShapeConfig:
    embed_dim: int = 512
    num_heads: int = 8
    head_dim: int = 0

    def __post_init__(self) -> None:
        require_positive(self.embed_dim, "embed_dim")
        require_positive(self.num_heads, "num_heads")
        if self.embed_dim % self.num_heads != 0:
            raise ConfigurationError(f"embed_dim ({self.embed_dim}) must be divisible by num_heads ({self.num_heads})",
                                     {"embed_dim": self.embed_dim, "num_heads": self.num_heads})


@dataclass(frozen=True, slots=True)
class AVQConfig:
    """Top-level immutable configuration."""

    attention: AttentionShapeConfig = field(default_factory=AttentionShapeConfig)
    codebook: CodebookConfig = field(default_factory=CodebookConfig)
    routing: RoutingConfig = field(default_factory=RoutingConfig)
    refinement: RefinementConfig = field(default_factory=RefinementConfig)
    merge: MergeConfig = field(default_factory=MergeConfig)
    backend: BackendConfig = field(default_factory=BackendConfig)
    cache: CacheConfig = field(default_factory=CacheConfig)
    precision: PrecisionConfig = field(default_factory=PrecisionConfig)
    execution: ExecutionConfig = field(default_factory=ExecutionConfig)
    hopfield: HopfieldConfig = field(default_factory=HopfieldConfig)
    dropout: float = 0.0
    causal: bool = False
    tolerance_atol: float = 1e-5
    tolerance_rtol: float = 1e-5

    def __post_init__(self) -> None:
        require_in_range(self.dropout, 0.0, 1.0, "dropout")
        require_positive(self.tolerance_atol, "tolerance_atol")
        require_positive(self.tolerance_rtol, "tolerance_rtol")
        if self.attention.head_dim == 0:
            object.__setattr__(self, "attention", AttentionShapeConfig(
                embed_dim=self.attention.embed_dim, num_heads=self.attention.num_heads,
                head_dim=self.attention.embed_dim // self.attention.num_heads))

    # -- serialisation (same schema as the reference) -----------------------

    def to_dict(self) -> dict[str, object]:
        out: dict[str, object] = {"schema_version": SCHEMA_VERSION}
        for f in fields(self):
            value = getattr(self, f.name)
            out[f.name] = asdict(value) if dataclasses.is_dataclass(value) else value
        return out

    @classmethod
    def from_dict(cls, data: dict[str, object] | object) -> AVQConfig:
        if not isinstance(data, dict):
            raise ConfigurationError(f"AVQConfig.from_dict expected dict, got {type(data).__name__}")
        schema = data.get("schema_version")
        if schema is not None and schema != SCHEMA_VERSION:
            raise ConfigurationError(f"AVQConfig schema_version mismatch: expected {SCHEMA_VERSION!r}, got {schema!r}",
                                     {"schema_version": schema})
        known = {f.name: f for f in fields(cls)}
        for k in data:
            if k != "schema_version" and k not in known:
                raise ConfigurationError(f"AVQConfig.from_dict got unknown field {k!r}", {"unknown_field": k})
        kwargs: dict[str, object] = {}
        for name, f in known.items():
            if name not in data:
                continue
            value = data[name]
            if isinstance(value, dict):
                target = _SUBCONFIGS.get(name)
                if target is not None:
                    value = target(**value)
            kwargs[name] = value
        return cls(**kwargs)  # type: ignore[arg-type]

    def save_json(self, path: str | Path) -> Path:
        target = Path(path)
        target.parent.mkdir(parents=True, exist_ok=True)
        try:
            target.write_text(json.dumps(self.to_dict(), indent=2, sort_keys=True))
        except (OSError, TypeError) as exc:
            raise ConfigurationError(f"failed to write AVQConfig JSON to {target}", {"path": str(target)}) from exc
        return target

    @classmethod
    def load_json(cls, path: str | Path) -> AVQConfig:
        source = Path(path)
        try:
            data = json.loads(source.read_text())
        except OSError as exc:
            raise ConfigurationError(f"failed to read AVQConfig JSON from {source}", {"path": str(source)}) from exc
        except json.JSONDecodeError as exc:
            raise ConfigurationError(f"invalid JSON in AVQConfig file {source}: {exc.msg}",
                                     {"path": str(source)}) from exc
        return cls.from_dict(data)


_SUBCONFIGS = {
    "attention": AttentionShapeConfig, "codebook": CodebookConfig, "routing": RoutingConfig,
    "refinement": RefinementConfig, "merge": MergeConfig, "backend": BackendConfig, "cache": CacheConfig,
    "precision": PrecisionConfig, "execution": ExecutionConfig, "hopfield": HopfieldConfig,
}

__all__ = [
    "AVQConfig", "AttentionShapeConfig", "BACKEND_NAMES", "BackendConfig", "CacheConfig", "CodebookConfig",
    "DEFAULT_EMA_DECAY", "ExecutionConfig", "HopfieldConfig", "MergeConfig", "PrecisionConfig",
    "RefinementConfig", "RoutingConfig", "SCHEMA_VERSION", "require_in_range", "require_non_negative",
    "require_positive",
]
