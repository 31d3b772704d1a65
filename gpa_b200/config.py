"""``GPAConfig`` with the ``b200`` backend (fisalt/GPA src/gpa/attention.py:17-75).

Same fields, defaults (except ``backend``) and validation messages as the
reference.  The b200 backend implements the default reader; flags that select
other operators are rejected with ``ValueError`` rather than silently falling
back, in the style of the reference's own checks (attention.py:45-75).
"""
from __future__ import annotations

from dataclasses import dataclass

MAX_LEVELS = 8
MAX_WIDTH = 128
MAX_CHUNK = 64


@dataclass(frozen=True)
class GPAConfig:
    heads: int = 4
    key_dim: int = 32
    value_dim: int = 32
    slots: tuple[int, ...] = (16, 16, 16, 16)
    positional_mode: str = "gated"  # gated | moments | none
    query_scale: float = 1 / 16
    beta_init: float = .1
    beta_max: float = .9
    decay_init: float = .001
    relation_beta_init: float = .6
    relation_decay_init: float = .0001
    chunk_size: int = 1
    backend: str = "b200"
    execution: str = "reference"  # every schedule computes the same lagged model on b200
    read_scale: float = 1.
    shared_query_center: bool = False
    rsa_update: bool = False
    paper_product_read: bool = False
    control_dim: int = 0
    slot_feature: str = "linear"
    slot_scale: float = 4.
    balanced_bridge: bool = False
    relation_marginal: bool = False
    quadratic_features: bool = False
    learn_read_scale: bool = False

    def __post_init__(self):
        # reference checks, same conditions and messages (attention.py:46-73)
        if min(self.heads, self.key_dim, self.value_dim, self.chunk_size) <= 0:
            raise ValueError("dimensions and chunk_size must be positive")
        if self.control_dim < 0:
            raise ValueError("control_dim must be nonnegative")
        if self.slot_feature not in ("linear", "softmax", "tanh") or self.slot_scale <= 0:
            raise ValueError("slot_feature must be linear/softmax/tanh, slot_scale positive")
        if self.relation_marginal and not self.paper_product_read:
            raise ValueError("relation marginal correction needs product reading")
        if not self.slots or min(self.slots) <= 0:
            raise ValueError("slots must contain positive capacities")
        if self.positional_mode not in ("gated", "moments", "none"):
            raise ValueError("unknown positional_mode")
        if self.positional_mode == "moments" and self.key_dim % 2:
            raise ValueError("positional moments require even key_dim")
        if not 0 < self.beta_init < self.beta_max <= 1:
            raise ValueError("require 0 < beta_init < beta_max <= 1")
        if not 0 < self.relation_beta_init < 1:
            raise ValueError("relation_beta_init must be in (0,1)")
        if self.decay_init <= 0 or self.relation_decay_init <= 0:
            raise ValueError("initial decays must be positive")
        if self.backend != "b200":
            raise ValueError("backend must be b200 (use the reference package for torch/fla)")
        if self.execution not in ("reference", "packed", "triton", "staged"):
            raise ValueError("execution must be reference, packed, triton, or staged")
        if self.read_scale <= 0:
            raise ValueError("read_scale must be positive")
        if self.shared_query_center and self.query_scale <= 0:
            raise ValueError("shared query-center parameterization needs query_scale > 0")
        # b200 operator coverage
        unsupported = [name for name, on in (
            ("rsa_update", self.rsa_update),
            ("control_dim", self.control_dim != 0),
            ("slot_feature!='linear'", self.slot_feature != "linear"),
            ("balanced_bridge", self.balanced_bridge),
            ("quadratic_features", self.quadratic_features),
            ("learn_read_scale", self.learn_read_scale),
            ("shared_query_center", self.shared_query_center),
        ) if on]
        if unsupported:
            raise ValueError("the b200 backend does not implement: " + ", ".join(unsupported))
        if self.chunk_size > MAX_CHUNK:
            raise ValueError(f"the b200 backend needs chunk_size <= {MAX_CHUNK}")
        if len(self.slots) > MAX_LEVELS:
            raise ValueError(f"the b200 backend supports at most {MAX_LEVELS} levels")
        if max(self.key_dim, self.value_dim, *self.slots) > MAX_WIDTH:
            raise ValueError(f"the b200 backend needs key_dim, value_dim and slots <= {MAX_WIDTH}")
