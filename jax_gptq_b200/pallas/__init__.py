from .blocked_pivoted_qr import blocked_pivoted_qr

__all__ = ["blocked_pivoted_qr"]
