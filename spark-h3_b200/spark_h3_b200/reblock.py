"""Landmark-tree-v2 reblocking on the B200: the per-(batch, head) token permutations that
group similar queries and similar keys into 64-token blocks before Spark routing.

Host side of the reference's reblock path:
  * `hilbert_midpoint_sample_indices`  mahalanobis_kmeans.py:11-96 (Skilling 3-D Hilbert
    order, N/64 uniformly spaced samples; integer host logic, cached per grid)
  * `initial_token_indices`            landmark_initial_order.py:44-77 (root orders)
  * `ReblockPlan`                      landmark_tree_v2.py:904-1172
    (PreparedLandmarkTreeV2Permutation: the hierarchy's node tables and scratch, prepared
    once per shape and reused)
  * `spark_reblock`                    spark.py:32 / landmark_tree_v2.py:835-901
    (recursive_landmark_tree_v2_blocks), default options only
  * `qk_block_permutations`            spark_integration.py:394-851
    (_landmark_tree_v2_qk_block_permutations: metric factors, [K.Lq ; Q.Lk] features, tree)
All device work runs in libsparkh3b200.so (sb_reblock_metric / _transform / _tree).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from functools import lru_cache

import numpy as np
import torch

from . import _lib
from .hierarchy import ReblockHierarchy, build_reblock_hierarchy
from .ops import _dtype_code, _require_cuda, _stream

INITIAL_ORDERS = ("flat", "tile_t4h4w4", "hilbert_thw", "hilbert_twh", "hilbert_htw", "hilbert_hwt", "hilbert_wth",
                  "hilbert_wht")
BLOCK = 64


def _grid_tuple(grid_shape) -> tuple[int, int, int]:
    if not isinstance(grid_shape, (tuple, list)) or len(grid_shape) != 3:
        raise ValueError("grid_shape must contain three positive integers (T,H,W)")
    grid = tuple(int(g) for g in grid_shape)
    if any(g <= 0 for g in grid):
        raise ValueError("grid_shape must contain three positive integers (T,H,W)")
    return grid


def _hilbert_index(coords: np.ndarray, bits: int) -> np.ndarray:
    """Hilbert index of [N, 3] integer coordinates on a 2^bits cube (Skilling's transpose:
    inverse-undo of the Gray-code excess, then bit interleaving, axis 0 most significant)."""
    x = coords.astype(np.int64, copy=True)
    top = 1 << (bits - 1)
    q = top
    while q > 1:
        mask = q - 1
        for axis in range(3):
            hi = (x[:, axis] & q) != 0
            x[hi, 0] ^= mask
            lo = ~hi
            t = (x[lo, 0] ^ x[lo, axis]) & mask
            x[lo, 0] ^= t
            x[lo, axis] ^= t
        q >>= 1
    x[:, 1] ^= x[:, 0]
    x[:, 2] ^= x[:, 1]
    gray = np.zeros(len(x), dtype=np.int64)
    q = top
    while q > 1:
        gray[(x[:, 2] & q) != 0] ^= q - 1
        q >>= 1
    x ^= gray[:, None]
    index = np.zeros(len(x), dtype=np.int64)
    for bit in range(bits - 1, -1, -1):
        for axis in range(3):
            index = (index << 1) | ((x[:, axis] >> bit) & 1)
    return index


@lru_cache(maxsize=32)
def _initial_order(grid: tuple[int, int, int], name: str) -> np.ndarray:
    frames, height, width = grid
    ids = np.arange(frames * height * width, dtype=np.int64)
    if name == "flat":
        return ids
    t, h, w = ids // (height * width), (ids // width) % height, ids % width
    if name == "tile_t4h4w4":
        tile = ((t // 4) * ((height + 3) // 4) + h // 4) * ((width + 3) // 4) + w // 4
        return np.argsort(tile * 64 + (t % 4) * 16 + (h % 4) * 4 + w % 4, kind="stable")
    axes = {"t": t, "h": h, "w": w}
    coords = np.stack([axes[a] for a in name[len("hilbert_"):]], axis=-1)
    bits = max(1, (max(grid) - 1).bit_length())
    return np.argsort(_hilbert_index(coords, bits), kind="stable")


def initial_token_indices(grid_shape, initial_order: str = "flat") -> np.ndarray:
    """Root order of the tree: raster ids in the named traversal (read-only, cached)."""
    if initial_order not in INITIAL_ORDERS:
        raise ValueError(f"initial_order must be one of {', '.join(INITIAL_ORDERS)}")
    return _initial_order(_grid_tuple(grid_shape), initial_order)


@lru_cache(maxsize=32)
def _midpoints(grid: tuple[int, int, int], count: int) -> np.ndarray:
    order = _initial_order(grid, "hilbert_thw")
    n = len(order)
    count = min(max(1, int(count)), n)
    pos = np.floor((np.arange(count, dtype=np.float64) + 0.5) * n / count).astype(np.int64)
    return order[np.minimum(pos, n - 1)]


def hilbert_midpoint_sample_indices(grid_shape, count: int) -> np.ndarray:
    """`count` token ids uniformly spaced along the 3-D Hilbert order of the grid; with
    count = N // 64 the middle token of every Hilbert block of 64."""
    return _midpoints(_grid_tuple(grid_shape), int(count))


def _schedule(hierarchy: ReblockHierarchy) -> np.ndarray:
    words = [len(hierarchy.split_budgets)]
    for level in hierarchy.split_budgets:
        words.append(len(level))
        for leaves, budgets in level:
            words += [int(leaves), len(budgets), *map(int, budgets)]
    return np.asarray(words, dtype=np.int32)


class ReblockPlan:
    """Node tables of one (tokens, fanout schedule, grid, root order), prepared once and
    reused for every call of that shape; scratch is kept per row count."""

    def __init__(self, tokens: int, children=16, *, grid_shape=None, fanout_mode: str = "power_of_two_fanout",
                 final_fanout=None, root_fanout=None, initial_order: str = "flat", proxy_iterations: int = 2,
                 seed_rule: str = "farthest_pair", device=None):
        proxy_iterations, seed_rule = normalize_proxy_controls(proxy_iterations, seed_rule)
        if tokens < BLOCK:
            raise ValueError("landmark-tree-v2 requires at least 64 non-empty rows")
        grid = _grid_tuple(grid_shape) if grid_shape is not None else (1, 1, tokens)
        if math.prod(grid) != tokens:
            raise ValueError("grid_shape product must equal the token count")
        self.tokens = tokens
        self.grid = grid
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.hierarchy = build_reblock_hierarchy(tokens, children, grid_shape=grid, fanout_mode=fanout_mode,
                                                 final_fanout=final_fanout, root_fanout=root_fanout)
        schedule = _schedule(self.hierarchy)
        length = _lib.load().sb_reblock_plan(schedule.ctypes.data, len(schedule), tokens, None, 0)
        _lib.check(int(length), "sb_reblock_plan")
        self.plan_host = np.zeros(int(length), dtype=np.int32)
        _lib.check(int(_lib.load().sb_reblock_plan(schedule.ctypes.data, len(schedule), tokens,
                                                   self.plan_host.ctypes.data, int(length))), "sb_reblock_plan")
        _lib.check(int(_lib.load().sb_reblock_plan_proxy(self.plan_host.ctypes.data, proxy_iterations,
                                                         int(seed_rule == "endpoint_order"))), "sb_reblock_plan_proxy")
        self.proxy_iterations, self.seed_rule = proxy_iterations, seed_rule
        self.plan_device = torch.from_numpy(self.plan_host).to(self.device)
        order = initial_token_indices(grid, initial_order)
        self.initial_order = initial_order
        self.root = None if initial_order == "flat" else torch.from_numpy(order.astype(np.int32)).to(self.device)
        self.num_excluded = tokens % BLOCK
        self.active_tokens = tokens - self.num_excluded
        self._workspace: dict[int, torch.Tensor] = {}
        self._features: dict[int, torch.Tensor] = {}
        self._graphs: dict[int, tuple] = {}  # rows -> (graph, features, perm, inverse)
        self._eager_runs: dict[int, int] = {}

    def workspace(self, rows: int) -> torch.Tensor:
        ws = self._workspace.get(rows)
        if ws is None:
            nbytes = int(_lib.load().sb_reblock_workspace_bytes(self.plan_host.ctypes.data, rows))
            _lib.check(nbytes, "sb_reblock_workspace_bytes")
            ws = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
            self._workspace[rows] = ws
        return ws

    def run(self, features: torch.Tensor, perm: torch.Tensor | None = None, inverse: torch.Tensor | None = None,
            excluded_indices: torch.Tensor | None = None):
        """features [rows, tokens, 128] bf16 (CUDA) -> (permutation, inverse) int32 [rows, tokens].
        excluded_indices [rows, tokens mod 64]: the protected remainder chosen by the caller
        instead of the largest-norm tokens (landmark_tree_clustering.py:99-119, same checks)."""
        if features.dim() != 3 or features.shape[1] != self.tokens:
            raise ValueError(f"features must be [rows, {self.tokens}, D]")
        if features.dtype != torch.bfloat16:
            raise RuntimeError("the CUDA landmark tree takes bf16 features")
        device = _require_cuda(features)
        rows, tokens, dim = features.shape
        frozen = None if excluded_indices is None else validate_excluded(excluded_indices, rows, tokens, device)
        if perm is None:
            perm = torch.empty((rows, tokens), dtype=torch.int32, device=device)
        if inverse is None:
            inverse = torch.empty((rows, tokens), dtype=torch.int32, device=device)
        ws = self.workspace(rows)
        root = None if self.root is None else self.root.data_ptr()
        with torch.cuda.device(device):
            if frozen is None:
                _lib.call("sb_reblock_tree", features.data_ptr(), rows, tokens, dim, root, self.plan_host.ctypes.data,
                          self.plan_device.data_ptr(), ws.data_ptr(), ws.numel(), perm.data_ptr(), inverse.data_ptr(),
                          _stream(device))
            else:
                _lib.call("sb_reblock_tree_frozen", features.data_ptr(), rows, tokens, dim, root, frozen.data_ptr(),
                          self.plan_host.ctypes.data, self.plan_device.data_ptr(), ws.data_ptr(), ws.numel(),
                          perm.data_ptr(), inverse.data_ptr(), _stream(device))
        return perm, inverse


    def features_buffer(self, rows: int) -> torch.Tensor:
        """The static features buffer [rows, tokens, 128] bf16 that replay() reads."""
        buf = self._features.get(rows)
        if buf is None:
            buf = torch.empty((rows, self.tokens, 128), dtype=torch.bfloat16, device=self.device)
            self._features[rows] = buf
        return buf

    def replay(self, rows: int) -> tuple[torch.Tensor, torch.Tensor]:
        """The tree over features_buffer(rows) as one CUDA graph launch, like the reference's
        prepared permutation (landmark_tree_v2.py:904-1172): the first call of a row count runs
        eagerly (module loading, kernel attributes), the second captures the launch sequence,
        later calls replay it.  Returns copies of (permutation, inverse) int32 [rows, tokens]."""
        features = self.features_buffer(rows)
        entry = self._graphs.get(rows)
        if entry is None:
            runs = self._eager_runs.get(rows, 0)
            if runs == 0:
                self._eager_runs[rows] = 1
                perm, inverse = self.run(features)
                return perm, inverse
            perm = torch.empty((rows, self.tokens), dtype=torch.int32, device=self.device)
            inverse = torch.empty_like(perm)
            self.workspace(rows)
            graph = torch.cuda.CUDAGraph()
            torch.cuda.current_stream(self.device).synchronize()
            with torch.cuda.device(self.device), torch.cuda.graph(graph):
                self.run(features, perm, inverse)
            entry = (graph, features, perm, inverse)
            self._graphs[rows] = entry
        graph, _, perm, inverse = entry
        graph.replay()
        return perm.clone(), inverse.clone()


@dataclass(frozen=True)
class LandmarkTreeV2Result:
    block_indices: torch.Tensor
    excluded_indices: torch.Tensor
    permutation: torch.Tensor
    inverse_permutation: torch.Tensor
    active_tokens: int
    num_excluded: int
    hierarchy: ReblockHierarchy


_PLANS: dict[tuple, ReblockPlan] = {}


def remainder_ids(features: torch.Tensor) -> torch.Tensor:
    """The protected remainder of bf16 features [rows, tokens, 128]: the tokens mod 64 ids of
    largest squared norm per row, equal norms to the lower id, ascending
    (landmark_tree_clustering.py:56-82), int32 [rows, tokens mod 64]."""
    device = _require_cuda(features)
    rows, tokens, dim = features.shape
    excluded = torch.empty((rows, tokens % BLOCK), dtype=torch.int32, device=device)
    workspace = torch.empty(8 * rows * tokens, dtype=torch.uint8, device=device)
    with torch.cuda.device(device):
        _lib.call("sb_reblock_remainder", features.contiguous().data_ptr(), rows, tokens, dim, workspace.data_ptr(),
                  workspace.numel(), excluded.data_ptr(), _stream(device))
    return excluded


def _required_m2_side(m2_side: str, layout_reuse: str) -> str:
    """The feature sides that take the opposite side's second moment, given the layouts that
    are built (spark_integration.py:365-380)."""
    if m2_side not in ("both", "query", "key", "none"):
        raise ValueError("m2_side must be both, query, key, or none")
    if layout_reuse == "independent":
        return m2_side
    if layout_reuse == "q_from_k":
        return "key" if m2_side in ("both", "key") else "none"
    return "query" if m2_side in ("both", "query") else "none"


def validate_excluded(excluded_indices, rows: int, tokens: int, device) -> torch.Tensor:
    """The caller's protected remainder, checked as landmark_tree_clustering.py:104-114 checks
    it (same messages): shape (rows, tokens mod 64), ids in range, unique per row.  Returns
    int32 ids on the device."""
    remainder = tokens % BLOCK
    excluded = torch.as_tensor(excluded_indices).to(device=device, dtype=torch.long)
    if tuple(excluded.shape) != (rows, remainder):
        raise ValueError(f"excluded_indices must have shape {(rows, remainder)}")
    if remainder:
        if bool(((excluded < 0) | (excluded >= tokens)).any()):
            raise ValueError("excluded_indices must lie in the original token range")
        ordered = excluded.sort(1).values
        if bool((ordered[:, 1:] == ordered[:, :-1]).any()):
            raise ValueError("excluded_indices must be unique per batch row")
    return excluded.to(torch.int32).contiguous()


def normalize_proxy_controls(proxy_iterations, seed_rule, update_rule="mean"):
    """The proxy controls of landmark_v2_terminal.py:43-50 (_normalize_proxy_controls), same
    messages.  The medoid update is refused: its choice between the two landmarks of a
    two-landmark side is an exact tie in real arithmetic, and the reference settles it by the
    rounding of its BLAS distance products, which no other arithmetic reproduces (on the
    reference's own fixtures, 31-39 % of permutation positions agreed)."""
    if type(proxy_iterations) is not int or proxy_iterations not in (0, 1, 2, 4):
        raise ValueError("proxy_iterations must be 0, 1, 2, or 4")
    if seed_rule not in ("farthest_pair", "endpoint_order"):
        raise ValueError("seed_rule must be farthest_pair or endpoint_order")
    if update_rule not in ("mean", "medoid"):
        raise ValueError("update_rule must be mean or medoid")
    if update_rule != "mean":
        raise NotImplementedError("the B200 landmark tree implements update_rule='mean' only")
    return proxy_iterations, seed_rule


def _plan(tokens, children, grid, fanout_mode, final_fanout, root_fanout, initial_order, device,
          proxy_iterations: int = 2, seed_rule: str = "farthest_pair") -> ReblockPlan:
    key = (tokens, children if isinstance(children, int) else tuple(children), grid, fanout_mode, final_fanout,
           root_fanout, initial_order, proxy_iterations, seed_rule, str(device))
    plan = _PLANS.get(key)
    if plan is None:
        plan = ReblockPlan(tokens, children, grid_shape=grid, fanout_mode=fanout_mode, final_fanout=final_fanout,
                           root_fanout=root_fanout, initial_order=initial_order, proxy_iterations=proxy_iterations,
                           seed_rule=seed_rule, device=device)
        _PLANS[key] = plan
    return plan


_DEFAULTS = dict(distance="cosine", order_mode="parent_order", group_size=1, fitting_samples=None,
                 landmark_mode="midpoint", landmark_count=32, midpoint_direction_mode="legacy", aggregation="linear",
                 proxy_iterations=2, seed_rule="farthest_pair", update_rule="mean", excluded_indices=None)


def spark_reblock(samples: torch.Tensor, *, grid_shape, initial_order: str = "flat", validate: bool = True,
                  max_children=16, fanout_mode: str = "power_of_two_fanout", fanout=None, final_fanout=None,
                  root_fanout=None, **options) -> LandmarkTreeV2Result:
    """Strict 64-token leaves of bf16 samples [..., N, 128] (landmark_tree_v2.py:835-901).

    Implements the production defaults (cosine distance, single tokens, 32 midpoint
    landmarks, linear aggregation, parent order) with every fanout mode of
    reblock_hierarchy.py (power_of_two_fanout, arbitrary_fanout, power_of_two_arbitrary_final:
    nodes of 2 to 64 children, split over landmark_v2_terminal.py's breadth-first topology),
    the proxy controls proxy_iterations (0, 1, 2, 4) and seed_rule (farthest_pair,
    endpoint_order) with mean updates, and a caller-chosen protected remainder
    (excluded_indices [rows, N mod 64]); other options raise NotImplementedError."""
    for name in options:
        if name not in _DEFAULTS:
            raise TypeError(f"spark_reblock() got an unexpected keyword argument {name!r}")
    proxy_iterations, seed_rule = normalize_proxy_controls(
        options.pop("proxy_iterations", 2), options.pop("seed_rule", "farthest_pair"),
        options.pop("update_rule", "mean"))
    excluded_indices = options.pop("excluded_indices", None)
    for name, value in options.items():
        default = _DEFAULTS[name]
        if (value is not default) and value != default:
            raise NotImplementedError(f"the B200 landmark tree implements {name}={default!r} only")
    if samples.ndim < 2 or not samples.is_floating_point():
        raise ValueError("samples must be floating point with layout [...,N,D]")
    leading = samples.shape[:-2]
    tokens, dim = samples.shape[-2:]
    if tokens < BLOCK or dim <= 0:
        raise ValueError("landmark-tree-v2 requires at least 64 non-empty rows")
    if samples.is_cuda and samples.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("CUDA landmark-tree-v2 requires FP16 or BF16 input")
    if dim != 128:
        raise NotImplementedError("the B200 landmark tree takes 128-dimensional features")
    children = fanout if fanout is not None else max_children
    flat = samples.reshape(-1, tokens, dim).to(torch.bfloat16).contiguous()
    plan = _plan(tokens, children, _grid_tuple(grid_shape), fanout_mode, final_fanout, root_fanout, initial_order,
                 flat.device, proxy_iterations, seed_rule)
    perm, inverse = plan.run(flat, excluded_indices=excluded_indices)
    perm64, inv64 = perm.long(), inverse.long()
    active = plan.active_tokens
    return LandmarkTreeV2Result(
        block_indices=perm64[:, :active].reshape(*leading, active // BLOCK, BLOCK),
        excluded_indices=perm64[:, active:].reshape(*leading, plan.num_excluded),
        permutation=perm64.reshape(*leading, tokens),
        inverse_permutation=inv64.reshape(*leading, tokens),
        active_tokens=active, num_excluded=plan.num_excluded, hierarchy=plan.hierarchy)


def metric_factors(q: torch.Tensor, k: torch.Tensor, samples: torch.Tensor, ridge: float = 1e-3) -> torch.Tensor:
    """Cholesky factors [2*B*H, 128, 128] fp32: rows [0, BH) from the sampled Q moments
    (applied to K), rows [BH, 2BH) from the sampled K moments (applied to Q)."""
    device = _require_cuda(q, k, samples)
    B, T, H, D = q.shape
    factors = torch.empty((2 * B * H, D, D), dtype=torch.float32, device=device)
    with torch.cuda.device(device):
        _lib.call("sb_reblock_metric", q.data_ptr(), k.data_ptr(), _dtype_code(q), B, T, H, D, samples.data_ptr(),
                  samples.numel(), float(ridge), factors.data_ptr(), _stream(device))
    return factors


def transform(q: torch.Tensor, k: torch.Tensor, factors: torch.Tensor, video_tokens: int,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """Reblock features [2*B*H, video, 128] bf16 = [K . bf16(Lq) ; Q . bf16(Lk)]."""
    device = _require_cuda(q, k, factors, out)
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16:
        raise RuntimeError("the reblock transform takes bf16 Q/K")
    B, T, H, D = q.shape
    shape = (2 * B * H, video_tokens, D)
    if out is not None and (tuple(out.shape) != shape or out.dtype != torch.bfloat16 or not out.is_contiguous()):
        raise ValueError(f"out must be contiguous bf16 {shape}")
    features = torch.empty(shape, dtype=torch.bfloat16, device=device) if out is None else out
    with torch.cuda.device(device):
        _lib.call("sb_reblock_transform", q.data_ptr(), k.data_ptr(), B, T, H, D, video_tokens, factors.data_ptr(),
                  features.data_ptr(), _stream(device))
    return features


_SAMPLES: dict[tuple, torch.Tensor] = {}


def qk_block_permutations(q: torch.Tensor, k: torch.Tensor, video_tokens: int, grid, *, children=16,
                          fanout_mode: str = "power_of_two_fanout", final_fanout=None, root_fanout=None,
                          ridge: float = 1e-3, initial_order: str = "flat", use_graph: bool = True,
                          proxy_iterations: int = 2, seed_rule: str = "farthest_pair",
                          layout_reuse: str = "independent", m2_side: str = "both"):
    """Paired opposite-second-moment Q/K permutations (spark_integration.py:394-851):
    returns (q_perm, q_inv, k_perm, k_inv), int32 [B, H, video], plus the reblock hierarchy.

    layout_reuse (spark_integration.py:365-380, 562-585, 725-729): "independent" builds a tree
    for K (features K . Lq) and one for Q (features Q . Lk); "q_from_k" builds only K's and Q
    takes the same permutation; "k_from_q" builds only Q's and K takes it.  With use_graph the
    independent trees replay a captured CUDA graph over the plan's static features buffer
    (the transform writes into it); a shared layout runs its one tree eagerly.

    m2_side (landmark_tree_v2_m2_side; spark_integration.py:450-466, 562-585, 597-693): which
    feature sides take the opposite side's second-moment factor -- "both", "key" (K . Lq
    only), "query" (Q . Lk only) or "none"; a side without it clusters its raw rows.  When the
    video leaves a remainder, the protected tail is frozen to the one the baseline (both-side)
    features choose, so the ablation does not change which tokens stay exact."""
    if layout_reuse not in ("independent", "q_from_k", "k_from_q"):
        raise ValueError(f"unknown layout reuse mode: {layout_reuse}")
    required = _required_m2_side(m2_side, layout_reuse)
    device = _require_cuda(q, k)
    B, T, H, D = q.shape
    grid = _grid_tuple(grid)
    key = (grid, video_tokens // BLOCK, str(device))
    samples = _SAMPLES.get(key)
    if samples is None:
        ids = hilbert_midpoint_sample_indices(grid, video_tokens // BLOCK)
        samples = torch.from_numpy(ids.astype(np.int32)).to(device)
        _SAMPLES[key] = samples
    factors = metric_factors(q, k, samples, ridge)
    plan = _plan(video_tokens, children, grid, fanout_mode, final_fanout, root_fanout, initial_order, device,
                 proxy_iterations, seed_rule)
    BH = B * H
    shape = (B, H, video_tokens)
    baseline = "both" if layout_reuse == "independent" else ("key" if layout_reuse == "q_from_k" else "query")
    if required != baseline:
        # rows [0, BH) of the features are K . Lq, rows [BH, 2BH) Q . Lk; a side without its
        # factor takes its raw rows, after the baseline features have chosen the tail
        features = transform(q, k, factors, video_tokens)
        rows = slice(0, 2 * BH) if layout_reuse == "independent" else (
            slice(0, BH) if layout_reuse == "q_from_k" else slice(BH, 2 * BH))
        excluded = remainder_ids(features[rows]) if video_tokens % BLOCK else None
        if required in ("query", "none"):
            features[:BH] = k[:, :video_tokens].permute(0, 2, 1, 3).reshape(BH, video_tokens, D)
        if required in ("key", "none"):
            features[BH:] = q[:, :video_tokens].permute(0, 2, 1, 3).reshape(BH, video_tokens, D)
        perm, inverse = plan.run(features[rows], excluded_indices=excluded)
        if layout_reuse != "independent":
            perm, inverse = perm.view(shape), inverse.view(shape)
            return perm, inverse, perm, inverse, plan.hierarchy
        return (perm[BH:].view(shape), inverse[BH:].view(shape), perm[:BH].view(shape), inverse[:BH].view(shape),
                plan.hierarchy)
    if layout_reuse != "independent":
        # rows [0, BH) of the features are K . Lq, rows [BH, 2BH) Q . Lk
        features = transform(q, k, factors, video_tokens)
        source = features[:BH] if layout_reuse == "q_from_k" else features[BH:]
        perm, inverse = plan.run(source)
        perm, inverse = perm.view(shape), inverse.view(shape)
        return perm, inverse, perm, inverse, plan.hierarchy
    if use_graph:
        transform(q, k, factors, video_tokens, out=plan.features_buffer(2 * B * H))
        perm, inverse = plan.replay(2 * B * H)
    else:
        perm, inverse = plan.run(transform(q, k, factors, video_tokens))
    return (perm[BH:].view(shape), inverse[BH:].view(shape), perm[:BH].view(shape), inverse[:BH].view(shape),
            plan.hierarchy)
