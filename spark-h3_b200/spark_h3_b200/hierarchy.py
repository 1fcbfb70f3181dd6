"""Reblock hierarchy planning: how the video's 64-token leaves split, round by round.

Restates the planning rules of h3_sparse_attention/reblock_hierarchy.py:1-234 (fanout
schedules, power-of-two and balanced child budgets, per-round capacities) and the
global-frontier query topology of h3_sparse_attention/landmark_virtual_q.py:30-65.  The
rules must agree exactly because the capacities drive the landmark tree's token splits.
"""
from __future__ import annotations

from collections import Counter
from dataclasses import dataclass
from functools import lru_cache

FANOUTS = (2, 4, 8, 16, 32, 64)
FANOUT_MODES = ("power_of_two_fanout", "arbitrary_fanout", "power_of_two_arbitrary_final")
INITIAL_ORDERS = ("flat", "tile_t4h4w4", "hilbert_thw", "hilbert_twh", "hilbert_htw", "hilbert_hwt",
                  "hilbert_wth", "hilbert_wht")


def normalize_children(children):
    """A per-level fanout schedule (scalar: every level); landmark_tree_v2.py:258-266."""
    if type(children) is int and children in FANOUTS:
        return children
    if isinstance(children, (list, tuple)) and children and all(type(v) is int and v in FANOUTS for v in children):
        return tuple(children)
    raise ValueError("children must be 2, 4, 8, 16, 32 or 64, or a nonempty list/tuple of those integers")


def normalize_fanout(max_children, fanout):
    if fanout is not None:
        if max_children != 16 and normalize_children(max_children) != normalize_children(fanout):
            raise ValueError("use fanout or legacy max_children, not conflicting values")
        max_children = fanout
    return normalize_children(max_children)


def normalize_order_mode(order_mode):
    if order_mode == "preserve_parent_order":
        return "parent_order"
    if order_mode not in ("parent_order", "scalar_order"):
        raise ValueError("order_mode must be parent_order or scalar_order")
    return order_mode


def normalize_group_size(group_size):
    if type(group_size) is int and group_size in (1, 2, 4, 8):
        return group_size
    if (isinstance(group_size, (list, tuple)) and group_size
            and all(type(v) is int and v in (1, 2, 4, 8) for v in group_size)):
        return tuple(group_size)
    raise ValueError("group_size must be 1, 2, 4 or 8, or a nonempty list/tuple of those integers")


def normalize_initial_order(initial_order):
    if initial_order not in INITIAL_ORDERS:
        raise ValueError(f"initial_order must be one of {', '.join(INITIAL_ORDERS)}")
    return initial_order


def normalize_fanout_mode(mode):
    if mode not in FANOUT_MODES:
        raise ValueError(f"fanout_mode must be one of {FANOUT_MODES}")
    return mode


def normalize_final_fanout(final_fanout):
    def ok(v):
        return type(v) is int and (2 <= v <= 32 or v == 64)
    if ok(final_fanout):
        return final_fanout
    if isinstance(final_fanout, (tuple, list)) and final_fanout and all(ok(v) for v in final_fanout):
        values = tuple(final_fanout)
        return values[0] if len(set(values)) == 1 else values
    raise ValueError("final_fanout must be an integer from 2 to 64 or a nonempty schedule")


def resolve_final_fanout(children, final_fanout=None, *, fanout_mode="arbitrary_fanout", terminal_leaf_blocks=None):
    children = (children,) if isinstance(children, int) else tuple(children)
    if terminal_leaf_blocks is not None:
        if terminal_leaf_blocks not in (0, 16):
            raise ValueError("legacy terminal_leaf_blocks must be 0 or 16")
        if final_fanout is not None:
            raise ValueError("use final_fanout or legacy terminal_leaf_blocks, not both")
    if fanout_mode == "power_of_two_fanout":
        inherited = normalize_final_fanout(children)
        if final_fanout is not None and normalize_final_fanout(final_fanout) != inherited:
            raise ValueError("a separate final_fanout requires arbitrary_fanout or power_of_two_arbitrary_final mode")
        return inherited
    if final_fanout is not None:
        return normalize_final_fanout(final_fanout)
    if terminal_leaf_blocks is not None:
        return normalize_final_fanout(tuple(max(c, terminal_leaf_blocks) for c in children))
    return normalize_final_fanout(children)


def resolve_root_fanout(children, root_fanout=None):
    if root_fanout is None:
        root_fanout = children if isinstance(children, int) else children[0]
    if type(root_fanout) is not int or root_fanout not in FANOUTS:
        raise ValueError("root_fanout must be 2, 4, 8, 16, 32 or 64, or None")
    return root_fanout


def _at(schedule, depth):
    return schedule if isinstance(schedule, int) else schedule[min(depth, len(schedule) - 1)]


def _fanout_alias(children, fanout):
    if fanout is None:
        return children
    if children != (16,) and children != fanout:
        raise ValueError("use fanout or legacy children, not conflicting values")
    return fanout


def balanced_child_budgets(leaves, children, depth=0, final_fanout=None, *, root_fanout=None,
                           terminal_leaf_blocks=None):
    """Fewest remaining rounds, then the smallest fanout that fits them; capacities differ by
    at most one leaf, largest first."""
    final_fanout = resolve_final_fanout(children, final_fanout, terminal_leaf_blocks=terminal_leaf_blocks)
    root_fanout = resolve_root_fanout(children, root_fanout)
    if leaves == 1:
        return (1,)
    if leaves <= _at(final_fanout, depth):
        return (1,) * leaves

    def limit(level):
        return root_fanout if level == 0 else children[min(level, len(children) - 1)]

    rounds = 1
    while True:
        capacity = _at(final_fanout, depth + rounds - 1)
        for level in range(depth + rounds - 2, depth - 1, -1):
            capacity *= limit(level)
        if capacity >= leaves:
            break
        rounds += 1
    if rounds == 1:
        count = leaves
    else:
        child_capacity = _at(final_fanout, depth + rounds - 1)
        for level in range(depth + rounds - 2, depth, -1):
            child_capacity *= limit(level)
        count = max(2, -(-leaves // child_capacity))
    q, r = divmod(leaves, count)
    return (q + 1,) * r + (q,) * (count - r)


def power_of_two_child_budgets(leaves, children, depth=0, *, root_fanout=None):
    """The largest power-of-two child count within the level's fanout, halving capacities
    (larger half first) until there are that many children."""
    if leaves < 2:
        return (1,)
    limit = resolve_root_fanout(children, root_fanout) if depth == 0 else children[min(depth, len(children) - 1)]
    count = 1
    while count * 2 <= min(leaves, limit):
        count *= 2
    frontier = (int(leaves),)
    while len(frontier) < count:
        frontier = tuple(v for budget in frontier for v in ((budget + 1) // 2, budget // 2))
    return frontier


@lru_cache(maxsize=64)
def tree_frontiers(leaves, children=(16,), roots=None, final_fanout=None, fanout_mode="power_of_two_fanout", *,
                   fanout=None, root_fanout=None, terminal_leaf_blocks=None):
    """Every level's frontier of leaf intervals, from the roots down to single leaves."""
    fanout_mode = normalize_fanout_mode(fanout_mode)
    children = _fanout_alias(children, fanout)
    if leaves < 1:
        raise ValueError("at least one complete video leaf is required")
    if isinstance(children, int):
        children = (children,)
    if not children or any(c not in FANOUTS for c in children):
        raise ValueError("invalid LMv2 child schedule")
    final_fanout = resolve_final_fanout(children, final_fanout, fanout_mode=fanout_mode,
                                        terminal_leaf_blocks=terminal_leaf_blocks)
    root_fanout = resolve_root_fanout(children, root_fanout)
    frontier = ((0, leaves),) if roots is None else tuple(roots)
    if (not frontier or frontier[0][0] != 0 or frontier[-1][1] != leaves
            or any(a >= b for a, b in frontier) or any(x[1] != y[0] for x, y in zip(frontier, frontier[1:]))):
        raise ValueError("roots must partition all video leaves in order")
    levels = [((0, leaves),), frontier] if roots is not None and len(frontier) > 1 else [frontier]
    depth = 0
    while any(b - a > 1 for a, b in frontier):
        nxt = []
        for a, b in frontier:
            size = b - a
            if size == 1:
                nxt.append((a, b))
                continue
            if fanout_mode != "power_of_two_fanout" and size <= _at(final_fanout, depth):
                budgets = (1,) * size
            elif fanout_mode in ("power_of_two_fanout", "power_of_two_arbitrary_final"):
                budgets = power_of_two_child_budgets(size, children, depth, root_fanout=root_fanout)
            else:
                budgets = balanced_child_budgets(size, children, depth, final_fanout, root_fanout=root_fanout)
            offset = a
            for count in budgets:
                nxt.append((offset, offset + count))
                offset += count
        frontier = tuple(nxt)
        levels.append(frontier)
        depth += 1
    return tuple(levels)


@dataclass(frozen=True)
class ReblockHierarchy:
    video_tokens: int
    children: tuple
    levels: tuple
    roots: tuple
    split_budgets: tuple  # per splitting round: ((node size, child capacities), ...)
    final_fanout: object = None
    fanout_mode: str = "power_of_two_fanout"
    root_fanout: int | None = None

    def __post_init__(self):
        object.__setattr__(self, "final_fanout",
                           resolve_final_fanout(self.children, self.final_fanout, fanout_mode=self.fanout_mode))
        object.__setattr__(self, "root_fanout", resolve_root_fanout(self.children, self.root_fanout))

    @property
    def fanout(self):
        return self.children[0] if len(set(self.children)) == 1 else self.children

    def budgets(self, splitting_round, leaves):
        for size, budgets in self.split_budgets[splitting_round]:
            if size == leaves:
                return budgets
        raise ValueError("node is not part of the prepared reblocking hierarchy")

    def metadata(self):
        return dict(hierarchy_boundary="video root", hierarchy_source="reblock_plan", fanout=self.fanout,
                    root_fanout=self.root_fanout, final_fanout=self.final_fanout, fanout_mode=self.fanout_mode)


@lru_cache(maxsize=128)
def build_reblock_hierarchy(video_tokens, children=(16,), *, grid_shape=None, final_fanout=None,
                            fanout_mode="power_of_two_fanout", fanout=None, root_fanout=None,
                            terminal_leaf_blocks=None):
    fanout_mode = normalize_fanout_mode(fanout_mode)
    children = _fanout_alias(children, fanout)
    if isinstance(children, int):
        children = (children,)
    leaves = video_tokens // 64
    final_fanout = resolve_final_fanout(children, final_fanout, fanout_mode=fanout_mode,
                                        terminal_leaf_blocks=terminal_leaf_blocks)
    root_fanout = resolve_root_fanout(children, root_fanout)
    levels = tree_frontiers(leaves, children, final_fanout=final_fanout, fanout_mode=fanout_mode,
                            root_fanout=root_fanout)
    rounds = []
    for parents, kids in zip(levels, levels[1:]):
        by_size = {}
        ci = 0
        for a, b in parents:
            budgets = []
            while ci < len(kids) and kids[ci][0] < b:
                x, y = kids[ci]
                budgets.append(y - x)
                ci += 1
            if b - a > 1:
                prev = by_size.setdefault(b - a, tuple(budgets))
                assert prev == tuple(budgets)
        rounds.append(tuple(sorted(by_size.items())))
    return ReblockHierarchy(video_tokens, tuple(children), levels, ((0, leaves),), tuple(rounds), final_fanout,
                            fanout_mode, root_fanout)


@lru_cache(maxsize=128)
def virtual_query_layout(video_tokens, total_tokens, levels_up, children=(8, 4), *, grid_shape=None,
                         fanout_mode="power_of_two_fanout", hierarchy=None):
    """Query parents: the frontier `levels_up` rounds above the leaves (levels_up >= depth
    gives the single global video parent), then one 64-token parent per remaining token
    block.  Returns ranges, leaf_to_virtual and metadata (landmark_virtual_q.py:30-65)."""
    if not (64 <= video_tokens <= total_tokens) or type(levels_up) is not int or levels_up < 0:
        raise ValueError("requires 64<=video_tokens<=total_tokens and nonnegative integer levels_up")
    if hierarchy is None:
        hierarchy = build_reblock_hierarchy(video_tokens, children, grid_shape=grid_shape, fanout_mode=fanout_mode)
    if hierarchy.video_tokens != video_tokens:
        raise ValueError("hierarchy and video token count differ")
    levels = hierarchy.levels
    leaves = video_tokens // 64
    cut = leaves * 64
    selected = max(0, len(levels) - 1 - levels_up)
    active = tuple((64 * a, 64 * b) for a, b in levels[selected])
    tail = tuple((start, min(start + 64, total_tokens)) for start in range(cut, total_tokens, 64))
    ranges = active + tail
    mapping = [-1] * (-(-total_tokens // 64))
    for parent, (start, end) in enumerate(ranges):
        for leaf in range(start // 64, -(-end // 64)):
            mapping[leaf] = parent
    metadata = dict(
        hierarchy.metadata(), video_tokens=video_tokens, total_tokens=total_tokens, active_video_tokens=cut,
        video_leaves=leaves, children=list(hierarchy.children), selected_completed_split_levels=selected,
        total_split_levels=len(levels) - 1, active_virtual_blocks=len(active), total_virtual_blocks=len(ranges),
        active_size_counts=dict(sorted(Counter(b - a for a, b in active).items())),
        frontier_size_counts=[dict(sorted(Counter(64 * (b - a) for a, b in level).items())) for level in levels],
        tail_policy="active-video-excluded tokens and packed context keep physical64 query blocks",
        levels_up=levels_up, effective_levels_up=len(levels) - 1 - selected, selection_mode="levels_up",
        global_video_representative=selected == 0,
        convention="global frontier before the last levels_up splitting rounds; already terminal64 leaves retained")
    return dict(ranges=ranges, leaf_to_virtual=tuple(mapping), metadata=metadata)
