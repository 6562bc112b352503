"""Process groups that can be destroyed and rebuilt (colocated training with offload).

Every NCCL communicator holds device buffers for as long as it lives. In colocated mode the
trainer's data-parallel-side groups (DP, expert DP, CP, pipeline and tied-embedding groups)
sit idle while the rollout engine generates, so `--offload-train` destroys them before the
rollout and rebuilds them before training: the memory goes to the KV cache meanwhile. Groups
the in-process engine itself uses (TP, EP) are created with tag "rollout" and kept.

The registry records each group's creation (rank list, backend, tag) in creation order, which
is identical on every rank, so `reload` can call `new_group` collectively in the same order.
Objects keep referring to the old group objects; `reload` walks the given roots (the process
context, the model, the actor, ...) through attributes, dicts, lists and tuples of this
package's objects and swaps every reference to a destroyed group for its replacement.

Reference: miles/utils/reloadable_process_group.py (destroy / reload around actor sleep and
wake_up, backends/megatron_utils/actor.py:195-220). The reference wraps every group in a proxy
and patches the collectives; here the groups stay plain torch groups and their holders are
rebound instead.
"""
from __future__ import annotations

import torch.distributed as dist


class ReloadableGroups:
    def __init__(self):
        self.specs: list[dict] = []

    def new_group(self, ranks=None, backend=None, tag: str = "train"):
        """dist.new_group, recorded (collective over the world, like dist.new_group)."""
        g = dist.new_group(ranks, backend=backend)
        self.specs.append({"ranks": None if ranks is None else list(ranks), "backend": backend,
                           "tag": tag, "group": g, "old": None})
        return g

    @staticmethod
    def _member(g) -> bool:
        return g is not None and g is not dist.GroupMember.NON_GROUP_MEMBER

    def destroy(self, tags=("train",)) -> int:
        """Destroy this rank's groups with one of `tags`; returns how many it destroyed."""
        n = 0
        for sp in self.specs:
            if sp["tag"] not in tags or sp["group"] is None:
                continue
            g = sp["group"]
            if self._member(g):
                dist.destroy_process_group(g)
                n += 1
            sp["old"], sp["group"] = g, None
        return n

    def reload(self, roots=()) -> dict:
        """Re-create every destroyed group (collective, creation order) and rebind the
        references held by `roots`; returns {id(old group): new group}."""
        mapping = {}
        for sp in self.specs:
            if sp["group"] is not None:
                continue
            g = dist.new_group(sp["ranks"], backend=sp["backend"])
            if self._member(sp["old"]):
                mapping[id(sp["old"])] = g
            sp["group"], sp["old"] = g, None
        if mapping:
            rebind(roots, mapping)
        return mapping


def _walkable(v) -> bool:
    mod = type(v).__module__ or ""
    return isinstance(v, (dict, list, tuple)) or mod.startswith(("miles_b200", "__main__"))


def rebind(roots, mapping: dict) -> None:
    """Replace every reference to a key group (by id) inside `roots` with its mapped group."""
    seen: set[int] = set()

    def fix(v):
        return mapping.get(id(v), v)

    def visit(obj):
        if id(obj) in seen:
            return obj
        seen.add(id(obj))
        if isinstance(obj, dict):
            for k, v in list(obj.items()):
                nv = fix(v)
                if nv is not v:
                    obj[k] = nv
                elif _walkable(v):
                    obj[k] = visit(v)
            return obj
        if isinstance(obj, list):
            for i, v in enumerate(obj):
                nv = fix(v)
                obj[i] = nv if nv is not v else (visit(v) if _walkable(v) else v)
            return obj
        if isinstance(obj, tuple):
            items = [fix(v) if fix(v) is not v else (visit(v) if _walkable(v) else v) for v in obj]
            if all(a is b for a, b in zip(items, obj)):
                return obj
            return type(obj)(*items) if hasattr(obj, "_fields") else type(obj)(items)
        d = getattr(obj, "__dict__", None)
        if d is not None:
            visit(d)
        return obj

    for r in roots:
        visit(r)


REGISTRY = ReloadableGroups()
