"""Stand-in for the third-party ``toposort`` package, written from its public API.

``toposort(deps)`` takes ``{item: set(dependencies)}`` and yields successive
sets ("layers"): first every item with no unmet dependency, then every item
whose dependencies all lie in earlier layers, and so on (Kahn's algorithm,
layer by layer).  Items that only appear as dependencies are included, and a
self-dependency is ignored.  A cycle raises ``ValueError``.  Used by the
reference's linearize pass (autodiff/linearize.py:10) when generating fixtures.
"""


class CircularDependencyError(ValueError):
    pass


def toposort(deps):
    pending = {k: set(v) - {k} for k, v in deps.items()}
    for v in list(pending.values()):
        for d in v:
            if d not in pending:
                pending[d] = set()
    while pending:
        ready = {k for k, v in pending.items() if not v}
        if not ready:
            raise CircularDependencyError(f"cycle among {sorted(pending)[:8]}")
        yield ready
        pending = {k: v - ready for k, v in pending.items() if k not in ready}


def toposort_flatten(deps, sort=True):
    out = []
    for layer in toposort(deps):
        out.extend(sorted(layer) if sort else layer)
    return out
