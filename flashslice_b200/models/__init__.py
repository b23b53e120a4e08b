from .transolver import TokenTransformerBlock, Transolver, TransolverBlock

__all__ = ["Transolver", "TransolverBlock", "TokenTransformerBlock"]
