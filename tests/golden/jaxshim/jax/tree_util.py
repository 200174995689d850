"""``register_dataclass`` is a no-op outside of JAX tracing (test infrastructure)."""


def register_dataclass(cls=None, **_kwargs):
    if cls is None:
        return lambda c: c
    return cls
