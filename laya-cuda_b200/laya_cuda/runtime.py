"""Shape classes (placeholder; the Runtime shim follows)."""


def span(tokens):
    """Rows start at multiples of 16 tokens (runtime.py:15-17)."""
    return -(-tokens // 16) * 16
