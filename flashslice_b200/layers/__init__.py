from .basic import MLP
from .physics_attention import Physics_Attention_Irregular_Mesh

__all__ = ["MLP", "Physics_Attention_Irregular_Mesh"]
