"""Stand-in for the third-party ``toposort`` package, written from its public API.

``toposort(deps)`` takes ``{item: set(dependencies)}`` and yields successive
sets ("layers"): first every item with no unmet dependency, then every item
whose dependencies all lie in earlier layers, and so on (Kahn's algorithm,
layer by layer).  Items that only appear as dependencies are included, and a
self-dependency is ignored.  A cycle raises ``ValueError``.  Used by the
reference's linearize pass (autodiff/linearize.py:10) when generating fixtures.

Each layer set is built by inserting its items in the order of the input
mapping (items that only appear as dependencies after all keys, in first-seen
order), so its iteration order is a function of the input alone.  The layers
are found with per-item counters of unmet dependencies (linear in the graph).
"""


class CircularDependencyError(ValueError):
    pass


def toposort(deps):
    order = {}
    for k in deps:
        order.setdefault(k, len(order))
    need = {k: set(v) - {k} for k, v in deps.items()}
    for v in list(need.values()):
        for d in v:
            if d not in need:
                order.setdefault(d, len(order))
                need[d] = set()
    items = list(order)
    users = {k: [] for k in items}
    for k, v in need.items():
        for d in v:
            users[d].append(k)
    left = {k: len(v) for k, v in need.items()}
    ready = [k for k in items if left[k] == 0]
    done = 0
    while ready:
        layer = set()
        for k in sorted(ready, key=order.__getitem__):
            layer.add(k)
        yield layer
        done += len(ready)
        nxt = []
        for k in ready:
            for u in users[k]:
                left[u] -= 1
                if left[u] == 0:
                    nxt.append(u)
        ready = nxt
    if done < len(items):
        pend = sorted(k for k in items if left[k] > 0)
        raise CircularDependencyError(f"cycle among {pend[:8]}")


def toposort_flatten(deps, sort=True):
    out = []
    for layer in toposort(deps):
        out.extend(sorted(layer) if sort else layer)
    return out
