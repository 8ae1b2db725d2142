"""Faster drop-ins for three passes of the reference front-end.

The reference front-end (graph -> kernalize -> linearize -> alloc) produces
the ``Proc`` this backend executes; three of its passes grow faster than
linearly with the graph and make large models untraceable.  ``install()``
replaces each by a function that returns the same result in the same order:

* ``fuse`` (linearize's greedy fusion), described below;
* ``_intern_repeat_opt`` (autodiff/opt/repeat_opt.py:12-62): the
  common-subexpression pass looks every node up in every duplicate group
  (building a set per group per node); here one id -> representative map,
  built in the same group order, answers each lookup;
* ``temp_alloc`` (autodiff/alloc/temp.py:12-35): marks buffers that live
  only inside one fused kernel as temporaries by calling
  ``change_to_temp(t)`` on every member for every such buffer; here each
  member's kernel arguments are visited once against the set of them.

The fusion pass.

The reference's ``linearize`` (autodiff/linearize.py:252-271) ends in
``fuse(block_id)`` (autodiff/linearize.py:103-249): a greedy fusion over the
block's topological layers.  For each fusion kind (DPElwFuse, ReduceElwFuse,
ElwFuse; autodiff/fusion/ops.py) it repeatedly opens a new group and scans the
layers from the first one: the first untaken node that can start a group
starts it, later nodes join it through ``FuseBase.attempt_fuse``
(autodiff/fusion/base.py:59-76), nodes that read the group but cannot join it
black-list everything downstream of them for the rest of the scan
(``get_walking_path``, autodiff/fusion/helper.py:70-81), and the scan stops
at the first layer, after the start, where nothing joined.

Every scan restarts at layer 0 and every black-listing walks all remaining
layers, so the pass grows with the cube of the graph: a per-(sequence, head)
transformer graph of 12 layers x 32 sequences x 16 heads would take more than
a day.  ``fuse`` below makes the same decisions in the same order, touching
only the nodes that can change the outcome:

* a scan starts directly at the first untaken node that can open a group
  (before a group is open, no other node has any effect);
* after the start only three kinds of nodes can act: readers of the group's
  results (pushed forward from each member through a consumer index), nodes
  downstream of a black-listed node (pushed forward the same way, layer by
  layer, instead of walking every later layer), and, for the horizontal
  ElwFuse (no dependency needed), the untaken elementwise nodes of the group's
  size.  They are visited in the reference's scan order (layer, then the
  layer set's iteration order); every other node would take the "no effect"
  branch of the reference loop;
* placing each finished group beside its last node uses an id -> layer index
  instead of a scan of all layers.

Groups are still built by the reference's own ``FuseBase`` objects, so member
order, fuse ids (one ``context.get_id()`` per opened scan) and the returned
``Proc`` are the reference's.  The shortcuts rely on one property of the
block's toposort: every dependency ``get_deps`` reports that is itself a node
of the block lies in an earlier layer.  ``fuse`` checks it and falls back to
the reference's function when it does not hold.

Use: ``ad_b200.frontend.install()`` once, after importing ``autodiff`` and
before ``autodiff.execute()``.
"""
from __future__ import annotations

from collections import defaultdict


def install() -> None:
    """Replace the three passes in the imported reference front-end."""
    temp_mod, lin, rep = _modules()
    if getattr(lin.fuse, "_ad_b200_fast", False):
        return
    orig = lin.fuse

    def fast(g_dep_id):
        return fuse(lin, orig, g_dep_id)

    fast._ad_b200_fast = True
    _saved.update(fuse=orig, repeat=rep._intern_repeat_opt, temp=temp_mod.temp_alloc)
    lin.fuse = fast
    rep._intern_repeat_opt = lambda context: intern_repeat_opt(rep, context)
    temp_mod.temp_alloc = temp_alloc


_saved = {}


def _modules():
    # by module path: ``autodiff.opt`` re-exports a function named ``repeat_opt``
    # that shadows the submodule of the same name as an attribute
    import importlib
    return tuple(importlib.import_module(m) for m in
                 ("autodiff.alloc.temp", "autodiff.linearize", "autodiff.opt.repeat_opt"))


def uninstall() -> None:
    temp_mod, lin, rep = _modules()
    if _saved:
        lin.fuse, rep._intern_repeat_opt, temp_mod.temp_alloc = _saved["fuse"], _saved["repeat"], _saved["temp"]
        _saved.clear()


def intern_repeat_opt(rep, context):
    """Same result as autodiff/opt/repeat_opt.py:12-62: group the nodes whose
    children and own parameters hash alike, then replace every later member
    of a group by its first member (the first group holding a node wins, as in
    the reference's linear search)."""
    groups = {}

    def track(node, _):
        if node.get_block() is not None:
            return node
        if isinstance(node, (rep.Tensor, rep.ConstantNode)):
            return node
        hs = tuple([ch.repeat_helper(is_child=True) for ch in node.children()]) + \
            tuple(node.repeat_helper(is_child=False))
        groups.setdefault(hs, []).append(node)
        return node

    context.procedure[0] = rep.walk_graph(context.procedure[0], track)
    dup = [nodes for nodes in groups.values() if len(nodes) > 1]
    first_of = {}
    for nodes in dup:
        for v in nodes[1:]:
            first_of.setdefault(v.id, nodes[0])

    def replace(node, _):
        return first_of.get(node.id, node)

    context.procedure[0] = rep.walk_graph(context.procedure[0], replace)
    return len(dup)


def temp_alloc(proc, fused_ids_to_of):
    """Same result as autodiff/alloc/temp.py:12-35."""
    from autodiff.alloc import AllocEntry, DeallocEntry
    from autodiff.node import Node
    for base in fused_ids_to_of.values():
        seen = {}
        for n in base.nodes:
            if isinstance(n, AllocEntry):
                seen[n.id] = False
            elif isinstance(n, DeallocEntry) and n.id in seen:
                seen[n.id] = True
        track = {i for i, both in seen.items() if both}
        if not track:
            continue
        for n in base.nodes:
            if isinstance(n, (AllocEntry, DeallocEntry)) and n.id in track:
                n.is_temp = True
            if isinstance(n, Node):
                for k in n.kargs:
                    _mark_temp(k, track)
                if not n.kres.is_none():
                    _mark_temp(n.kres, track)


def _mark_temp(k, track):
    """``KernelArg.change_to_temp`` for every id of ``track`` at once
    (autodiff/kernalize/__init__.py:70-72, 109-111, 127-128)."""
    if hasattr(k, "karg_one"):
        _mark_temp(k.karg_one, track)
        _mark_temp(k.karg_two, track)
    elif hasattr(k, "constant"):
        return
    elif k.id in track:
        k.is_temp = True


def fuse(lin, orig, g_dep_id):
    """Same result as autodiff/linearize.py:103-249 ``fuse(g_dep_id)``."""
    from autodiff.context import Proc
    from autodiff.fusion.base import FuseBase, FuseResult
    from autodiff.fusion.helper import get_deps, get_res
    from autodiff.fusion.ops import DPElwFuse, ElwFuse, ReduceElwFuse, calc_size, is_elw
    from autodiff.node import Node

    id_to_node = lin.id_to_node
    toposort_res = list(lin.toposort(lin.global_deps[g_dep_id]))

    # ---- indexes: scan order, dependencies (cached: linearize never changes a
    # node's kernel args), consumers
    layers = [list(layer) for layer in toposort_res]
    layer_of, pos_of = {}, {}
    for li, lst in enumerate(layers):
        for pi, nid in enumerate(lst):
            layer_of[nid] = li
            pos_of[nid] = pi
    deps_of = {nid: get_deps(id_to_node[nid]) for nid in layer_of}
    consumers = defaultdict(list)
    for nid, ds in deps_of.items():
        for d in ds:
            if d in layer_of:
                if layer_of[d] >= layer_of[nid]:
                    return orig(g_dep_id)      # precondition of the shortcuts does not hold
                consumers[d].append(nid)

    entries = []
    init_taken = set()
    for op in (DPElwFuse, ReduceElwFuse, ElwFuse):
        horizontal = op is ElwFuse
        starters = [nid for lst in layers for nid in lst if op._init(None, id_to_node[nid])]
        sp = 0
        elw_by_size = []
        if horizontal:
            for lst in layers:
                by = defaultdict(list)
                for nid in lst:
                    n = id_to_node[nid]
                    if is_elw(n):
                        by[calc_size(n)].append(nid)
                elw_by_size.append(by)
        while True:
            entry = op()
            while sp < len(starters) and starters[sp] in init_taken:
                sp += 1
            if sp == len(starters):
                break                      # nothing can open a group: empty entry
            first = starters[sp]
            _scan(entry, first, layers, layer_of, pos_of, deps_of, consumers, init_taken,
                  id_to_node, get_res, FuseResult, elw_by_size if horizontal else None, calc_size)
            if len(entry.nodes) == 1:
                init_taken.add(entry.nodes[0].id)
            elif len(entry.nodes) > 1:
                entries.append(entry)

    # ---- place each group in its last node's layer, drop the members
    removed = set()
    for entry in entries:
        li = layer_of.get(entry.nodes[-1].id)
        if li is None:
            raise Exception("Couldn't find node in toposort_res to insert fused entry")
        id_to_node[entry.fuse_id] = entry
        toposort_res[li].add(entry.fuse_id)
        for n in entry.nodes:
            removed.add(n.id)
    # (the set-building expressions below are kept as the reference writes them:
    # a set's iteration order depends on how it was built, and the final order
    # of the proc follows it)
    for li, layer in enumerate(toposort_res):
        toposort_res[li] = set(filter(lambda x: x not in removed, layer))

    # ---- inner blocks, result -> group id, re-toposort (as the reference)
    replace = {}
    for layer in toposort_res:
        for nid in layer:
            node = id_to_node[nid]
            if isinstance(node, Node) and (block := node.get_block()) is not None:
                node.proc = lin.fuse(block.id)
                replace.update({r: node.id for r in get_res(node, True)})
            if isinstance(node, FuseBase):
                replace.update({r: node.fuse_id for r in get_res(node)})
    g_dep = {}
    for layer in toposort_res:
        for nid in layer:
            node = id_to_node[nid]
            ds = get_deps(node, step_proc=True)
            ds = set({(replace[d] if d in replace else d) for d in ds})
            g_dep[node.id if isinstance(node, Node) else node.fuse_id] = ds
    for k in g_dep:
        g_dep[k] = set(filter(lambda x: x in g_dep.keys(), g_dep[k]))
    out = []
    for layer in list(lin.toposort(g_dep)):
        for nid in layer:
            out.append(id_to_node[nid])
    return Proc(out)


def _scan(entry, first, layers, layer_of, pos_of, deps_of, consumers, init_taken, id_to_node,
          get_res, FuseResult, elw_by_size, calc_size):
    """One scan of the reference's fusion loop (autodiff/linearize.py:128-170),
    starting at the node that opens the group."""
    tracker = entry.result_tracker
    readers = defaultdict(set)     # layer -> nodes reading a member of the group
    black_in = defaultdict(set)    # layer -> nodes downstream of a black-listed node
    black = set()

    def joined(nid):
        for r in get_res(id_to_node[nid]):
            for c in consumers.get(r, ()):
                readers[layer_of[c]].add(c)

    def blacklist(nid):
        black.add(nid)
        for c in consumers.get(nid, ()):
            black_in[layer_of[c]].add(c)

    r = entry.attempt_fuse(id_to_node[first])
    assert r == FuseResult.INIT
    init_taken.add(first)
    joined(first)
    L = layer_of[first]
    size = calc_size(id_to_node[first]) if elw_by_size is not None else None
    after = pos_of[first]
    while L < len(layers):
        for b in black_in.pop(L, ()):
            if b not in black:
                blacklist(b)
        cands = readers.pop(L, set())
        if elw_by_size is not None:
            lst = elw_by_size[L].get(size)
            if lst:
                keep = [x for x in lst if x not in init_taken]
                elw_by_size[L][size] = keep
                cands.update(keep)
        did = L == layer_of[first]
        for nid in sorted(cands, key=pos_of.__getitem__):
            if pos_of[nid] <= after:
                continue
            reads = not tracker.isdisjoint(deps_of[nid])
            if nid in init_taken:
                if reads:
                    blacklist(nid)
                continue
            if nid in black:
                continue
            res = entry.attempt_fuse(id_to_node[nid])
            if res in (FuseResult.ADD, FuseResult.INIT):
                init_taken.add(nid)
                did = True
                joined(nid)
            elif not tracker.isdisjoint(deps_of[nid]):
                blacklist(nid)
        if not did:
            break
        L += 1
        after = -1
