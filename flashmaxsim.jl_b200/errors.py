"""Exception types mirroring the Julia exceptions the reference raises."""


class DimensionMismatch(ValueError):
    """Shapes of features, masks, indices or cotangents disagree
    (Julia `DimensionMismatch`, e.g. forward_pair.jl:14-21)."""


class ArgumentError(ValueError):
    """An argument is not acceptable (Julia `ArgumentError`, e.g. colocation.jl:27-35,
    ka.jl:41-46, dispatch.jl:53-56)."""
