"""Packed token layout: target video first in THW raster order, all other tokens after.

Same contract as h3_sparse_attention/processor.py:537-688 (`PackedLayout` and
`_packed_layout`), including the structural target-suffix selection and the composite
ordering of heterogeneous conditioning grids.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass
class PackedLayout:
    permutation: torch.Tensor
    inverse_permutation: torch.Tensor
    grid: tuple
    video_tokens: int
    sequence_length: int
    video_positions: torch.Tensor
    target_video_tokens: int | None = None
    condition_video_tokens: int = 0
    sparse_video_scope: str = "target"


def _raster(position_ids: torch.Tensor, indices: torch.Tensor):
    """(positions, grid, order, dense): sort indices by (t, h, w) rank and report whether they
    fill the grid spanned by their distinct coordinates exactly once."""
    pos = position_ids.index_select(0, indices)
    axes = [pos[:, a].unique(sorted=True) for a in range(3)]
    grid = tuple(int(ax.numel()) for ax in axes)
    rank = [torch.searchsorted(axes[a], pos[:, a].contiguous()) for a in range(3)]
    key = (rank[0] * grid[1] + rank[1]) * grid[2] + rank[2]
    order = key.argsort()
    dense = key.numel() == math.prod(grid) and torch.equal(
        key.index_select(0, order), torch.arange(math.prod(grid), device=key.device))
    return pos, grid, order, dense


def _time_planes(position_ids: torch.Tensor, indices: torch.Tensor):
    """Raster order of a composite whose time planes may each use a different grid."""
    pos = position_ids.index_select(0, indices)
    parts = []
    for t in pos[:, 0].unique(sorted=True):
        plane = indices.index_select(0, torch.nonzero(pos[:, 0] == t, as_tuple=False).flatten())
        _, grid, order, dense = _raster(position_ids, plane)
        if not dense or grid[0] != 1:
            return None
        parts.append(plane.index_select(0, order))
    return torch.cat(parts)


def packed_layout(token_tags: torch.Tensor, position_ids: torch.Tensor, *, video_indices=None, timestep_indices=None,
                  text_indices=None, sparse_video_scope: str = "target") -> PackedLayout:
    if token_tags.ndim != 1 or position_ids.shape != (token_tags.numel(), 3):
        raise ValueError("H3 token_tags/position_ids have unexpected shapes")
    if video_indices is not None and timestep_indices is not None and text_indices is not None:
        if text_indices.numel() == 0:
            raise ValueError("packed H3 sequence contains no text row to identify target-video timestep")
        if video_indices.numel() == 0:
            raise ValueError("packed H3 sequence contains no video rows")
        # The generated target is the final contiguous run of video rows; conditioning video
        # (possibly sharing the target's timestep) precedes it.
        breaks = torch.nonzero(video_indices[1:] != video_indices[:-1] + 1, as_tuple=False).flatten()
        start = int(breaks[-1].item() + 1) if breaks.numel() else 0
        target = video_indices[start:]
        condition = video_indices[:start]
        if target[-1] != token_tags.numel() - 1:
            raise ValueError("H3 target video rows must be the final packed-sequence suffix")
        text_timestep = timestep_indices[text_indices[0]]
        if not bool((timestep_indices.index_select(0, target) == text_timestep).all()):
            raise ValueError("H3 target video timestep does not match the text timestep")
        if video_indices.numel() and not bool((token_tags.index_select(0, video_indices) == 0).all()):
            raise ValueError("H3 video_indices selected rows whose modality tag is not video")
        if sparse_video_scope == "target":
            video = target
        elif sparse_video_scope == "target_and_condition":
            video = video_indices
        else:
            raise ValueError("sparse_video_scope must be 'target' or 'target_and_condition'")
    else:
        video = torch.nonzero(token_tags == 0, as_tuple=False).flatten()
        target = video
        condition = video[:0]
        if sparse_video_scope != "target":
            raise ValueError("target_and_condition scope requires H3 video/timestep/text indices")
    if video.numel() == 0:
        raise ValueError("packed H3 sequence contains no video tokens")
    selected = torch.zeros(token_tags.numel(), device=token_tags.device, dtype=torch.bool)
    selected[video] = True
    others = torch.nonzero(~selected, as_tuple=False).flatten()

    pos, grid, order, dense = _raster(position_ids, video)
    if dense:
        ordered = video.index_select(0, order)
        ordered_pos = pos.index_select(0, order)
    elif sparse_video_scope == "target_and_condition" and condition.numel():
        # Conditioning and target grids differ: keep each segment raster-ordered and
        # contiguous, and expose a flat composite grid.
        segments = []
        for name, segment in (("condition", condition), ("target", target)):
            _, seg_grid, seg_order, seg_dense = _raster(position_ids, segment)
            if not seg_dense and name == "condition":
                composite = _time_planes(position_ids, segment)
                if composite is not None:
                    segments.append(composite)
                    continue
            if not seg_dense:
                raise ValueError(f"{name} video tokens do not form a dense grid: grid={seg_grid}, "
                                 f"rows={segment.numel()}")
            segments.append(segment.index_select(0, seg_order))
        ordered = torch.cat(segments)
        ordered_pos = position_ids.index_select(0, ordered)
        grid = (1, 1, video.numel())
    else:
        raise ValueError(f"video tokens do not form a dense grid: grid={grid}, rows={video.numel()}")
    permutation = torch.cat((ordered, others))
    inverse = torch.empty_like(permutation)
    inverse[permutation] = torch.arange(permutation.numel(), device=permutation.device)
    return PackedLayout(permutation=permutation, inverse_permutation=inverse, grid=grid, video_tokens=video.numel(),
                        sequence_length=token_tags.numel(), video_positions=ordered_pos,
                        target_video_tokens=target.numel(), condition_video_tokens=condition.numel(),
                        sparse_video_scope=sparse_video_scope)
