"""Host helpers of the tile language that the op surface needs (tilec/language.py:16-18)."""


def cdiv(a, b):
    """Ceiling division, for host code: cdiv(5000, 4096) == 2."""
    return (a + b - 1) // b
