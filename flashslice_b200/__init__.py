"""flashslice_b200: the slice/deslice coupling of Transolver's
physics-attention on B200 (sm_100a), a drop-in for the operator surface of
Shizheng-Wen/flashslice.

    from flashslice_b200 import Transolver
    model = Transolver(space_dim=3, fun_dim=1, out_dim=4, use_fused_slice=True)

    from flashslice_b200.kernels import fused_slice, fused_deslice, unsupported_dims

The ops run in hand-written CUDA kernels behind the C ABI of
``include/flashslice_b200.h`` (``flashslice_b200/_native/libflashslice_b200.so``,
built by ``python -m flashslice_b200.build``).
"""

from .layers.physics_attention import Physics_Attention_Irregular_Mesh
from .models.transolver import TokenTransformerBlock, Transolver, TransolverBlock

__all__ = ["Transolver", "TransolverBlock", "TokenTransformerBlock",
           "Physics_Attention_Irregular_Mesh"]
__version__ = "0.1.0"
