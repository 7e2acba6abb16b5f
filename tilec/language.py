"""tilec.language's host helper (tilec/language.py:16-18); the tile-language builtins the
reference's compiler consumes have no counterpart here (no run-time compiler)."""
from tilec_b200.language import cdiv  # noqa: F401

__all__ = ["cdiv"]
