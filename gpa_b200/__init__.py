"""B200-native DenseGPA attention core (fisalt/GPA ``gpa`` API, backend ``"b200"``).

    from gpa_b200 import DenseGPA, GPAConfig
    model = DenseGPA(GPAConfig(heads=16, key_dim=128, value_dim=128,
                               slots=(64, 64, 64, 128), chunk_size=64)).cuda()
    out, state = model(q, k, v)            # q, k, v: [B, T, H, D] CUDA tensors
    out2, state = model(q2, k2, v2, state)  # cached continuation / decode

The compute runs in ``libgpa_b200.so`` (hand-written sm_100a kernels behind
the C ABI of ``include/gpa_b200.h``).
"""
from .config import GPAConfig
from .core import DenseGPA, edges_of
from .state import GPAState, LevelState, RelationState, ResidualSnapshot, tensors

__all__ = ["DenseGPA", "GPAConfig", "GPAState", "LevelState", "RelationState",
           "ResidualSnapshot", "edges_of", "tensors"]
__version__ = "0.1.0"
