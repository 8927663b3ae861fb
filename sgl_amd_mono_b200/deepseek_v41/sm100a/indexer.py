"""K2i's host side on one rank (the role of the reference's ``gfx950/indexer/runner.py``):
buffers that a replayed graph reads, the step's walk plans, and an index source's selection
-- K2i's logits, then the top-k (ties to the lower position) written as the layer's sparse
raw / page indices. Three kinds, as the reference (``indexer/runner.py:10-20``):

- ``full``: score every visible column of each row, keep the top ``topk``.
- ``producer``: ``full``, and the rows' candidate blocks (top 2048 blocks of 8 columns by
  their largest logit), which the step's ``reindex`` layers read.
- ``reindex``: score only the candidate blocks' columns, keep the top ``topk`` of them, and
  map them back to positions and pool slots.
"""

from __future__ import annotations

import torch

from ...common import ext
from . import abi

PLANE_ROWS = 64
CHUNK = 128
TOPK_BLOCKS = 2048
BLOCK_ROWS = 8
COMPACT = TOPK_BLOCKS * BLOCK_ROWS
MAX_ROWS = 48
KINDS = ("full", "producer", "reindex")


def _p(t):
    return 0 if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def check_plane(payload: torch.Tensor, scale: torch.Tensor) -> None:
    """Raise unless the plane is the split FP4 layout of 64-row pages
    (``indexer/runner.py:63-79`` of the reference)."""
    u8 = payload.view(torch.uint8)
    pages = scale.shape[0]
    if not (u8.is_contiguous() and scale.is_contiguous() and scale.dtype == torch.uint8
            and u8.numel() == pages * 4 * PLANE_ROWS * 16 and scale.numel() == pages * 4 * PLANE_ROWS):
        raise RuntimeError(f"K2i index plane: payload {tuple(payload.shape)}, scales {tuple(scale.shape)}; "
                           f"want [pages, 1, 4, {PLANE_ROWS}, 16] and [pages, 1, 4, {PLANE_ROWS}] bytes")


class Candidates:
    """A producer's candidate blocks of each row: ``ids`` [rows, 2048], -1 after the kept."""

    def __init__(self, ids: torch.Tensor):
        self.ids = ids


class K2iRunner:
    def __init__(self, device: torch.device, bound_max: int, topk: int = 512, ctas: int | None = None):
        dev = torch.device(device)
        if ctas is None:
            # one scoring CTA an SM (the tensor-core scorer holds a whole SM's TMEM): measured at
            # config 3, 35.0 us against 39.2 us with two tasks an SM
            ctas = torch.cuda.get_device_properties(dev).multi_processor_count
        self.dev, self.topk, self.ctas = dev, topk, ctas
        f32 = dict(dtype=torch.float32, device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
        self.bound_max = -(-max(bound_max, COMPACT) // CHUNK) * CHUNK
        self.ilog = torch.empty(MAX_ROWS * self.bound_max, **f32)
        self.cand_in = torch.empty(MAX_ROWS, TOPK_BLOCKS, **i32)
        self.cand_ids = torch.empty(MAX_ROWS, TOPK_BLOCKS, **i32)
        self.cand_table = torch.empty(MAX_ROWS, TOPK_BLOCKS, **i32)
        self.cand_bound = torch.empty(MAX_ROWS, **i32)
        self.compact_pos = torch.empty(MAX_ROWS, topk, **i32)
        self.plans = {r: torch.zeros(ctas, 4, **i32) for r in (1, 2)}
        self._query: dict[int, tuple] = {}  # per index head count: q, qscale, w, scratch
        t = torch.arange(MAX_ROWS)
        self.owners = torch.stack([t // p * p for p in range(1, MAX_ROWS + 1)]).to(**i32)

    # ------------------------------------------------------------ query
    def query(self, *, q: torch.Tensor, cos_sin: torch.Tensor, pos: torch.Tensor, x: torch.Tensor,
              wp: torch.Tensor, scale: float) -> tuple:
        """The FP4 query of decode rows (``dsv41_index_query``) from wq_b's output q [rows,
        heads * 128] bf16, the layer's RoPE table, the rows' positions, their normed rows x and
        the head weight projection wp [heads, hidden] bf16 with its scale: (q [rows, heads, 64]
        E2M1 pairs, qscale [rows, 1, 4, 16, 4], w [rows, heads] bf16), views of buffers this
        runner keeps per head count (first call outside graph capture)."""
        import struct
        M, H, hidden = x.shape[0], wp.shape[0], x.shape[1]
        if q.dtype != torch.bfloat16 or q.numel() != M * H * 128 or not q.is_contiguous():
            raise RuntimeError(f"K2i query: wq_b output {tuple(q.shape)} {q.dtype}, want [{M}, {H * 128}] bf16")
        if x.dtype != torch.bfloat16 or wp.dtype != torch.bfloat16 or tuple(wp.shape) != (H, hidden):
            raise RuntimeError(f"K2i query: x {tuple(x.shape)} {x.dtype}, weights_proj {tuple(wp.shape)} {wp.dtype}")
        if H not in self._query:
            u8 = dict(dtype=torch.uint8, device=self.dev)
            self._query[H] = (torch.empty(MAX_ROWS, H, 64, **u8), torch.zeros(MAX_ROWS, 1, 4, 16, 4, **u8),
                              torch.empty(MAX_ROWS, H, dtype=torch.bfloat16, device=self.dev),
                              torch.empty(MAX_ROWS * H * 4, **u8))
        q_out, qscale, w_out, scratch = self._query[H]
        bits = struct.unpack("<I", struct.pack("<f", float(scale)))[0]
        a = abi.IndexQueryArgs(M=M, heads=H, dim=128, rope=cos_sin.shape[1], hidden=hidden, q=_p(q),
                               cos_sin=_p(cos_sin), rope_rows=cos_sin.shape[0], pos=_p(pos),
                               x=_p(x.contiguous()), wp=_p(wp.contiguous()), weight_scale_f32=bits,
                               q_out=_p(q_out), qscale=_p(qscale), w_out=_p(w_out), scratch=_p(scratch),
                               scratch_bytes=scratch.numel())
        ext.call("dsv41_index_query", a, _stream())
        return q_out[:M], qscale[:M], w_out[:M]

    # ------------------------------------------------------------ plan
    def walk_plan(self, *, ratio: int, bounds: torch.Tensor, rows: int, per_req: int) -> torch.Tensor:
        plan = self.plans[ratio]
        a = abi.WalkPlanArgs(rows=rows, ctas=self.ctas, topk=self.topk, bounds=_p(bounds),
                             owners=_p(self.owners[per_req - 1]), plan=_p(plan))
        ext.call("dsv41_walk_plan", a, _stream())
        return plan

    # ------------------------------------------------------------ scoring
    def _score(self, *, rows, query, plane, plan, itab, itab_stride, itab_len, entry_rows, owners, bounds,
               lstride, reindex, reindex_chunks=0, out=None):
        q, qs, w = query
        payload, scale = plane
        a = abi.K2iArgs(rows=rows, heads=q.shape[1], q=_p(q), qscale=_p(qs), w=_p(w), payload=_p(payload),
                        kscale=_p(scale), plan=_p(plan), ctas=self.ctas, itab=_p(itab), itab_stride=itab_stride,
                        itab_len=itab_len, entry_rows=entry_rows, owners=_p(owners), bounds=_p(bounds),
                        logits=_p(self.ilog if out is None else out), lstride=lstride, reindex=reindex,
                        reindex_chunks=reindex_chunks)
        ext.call("dsv41_k2i", a, _stream())

    def score(self, *, rows, per_req, ratio, query, plane, page_table, bounds) -> torch.Tensor:
        """A FULL or producer layer's logits [rows, width] f32, valid below each row's bound."""
        width = min(page_table.shape[1] * PLANE_ROWS, self.bound_max)
        self._score(rows=rows, query=query, plane=plane, plan=self.plans[ratio], itab=page_table,
                    itab_stride=page_table.stride(0), itab_len=page_table.shape[1], entry_rows=PLANE_ROWS,
                    owners=self.owners[per_req - 1], bounds=bounds, lstride=width, reindex=0)
        return self.ilog[: rows * width].view(rows, width)

    def score_candidates(self, *, candidates, rows, per_req, query, plane, page_table, bounds):
        """A REINDEX layer's logits of its candidate blocks' columns: (compact [rows, COMPACT],
        lens [rows], ids [rows, 2048] with the newest block last)."""
        if tuple(candidates.ids.shape) != (rows, TOPK_BLOCKS):
            raise RuntimeError(f"K2i: candidate blocks {tuple(candidates.ids.shape)} for {rows} rows")
        owners = self.owners[per_req - 1]
        ids, lens = self.cand_ids[:rows], self.cand_bound[:rows]
        a = abi.ReindexArgs(rows=rows, topk_blocks=TOPK_BLOCKS, units=PLANE_ROWS // BLOCK_ROWS,
                            block_rows=BLOCK_ROWS, ids=_p(candidates.ids), ids_stride=candidates.ids.stride(0),
                            page_table=_p(page_table), page_stride=page_table.stride(0), owners=_p(owners),
                            visible=_p(bounds), ids_out=_p(ids), table=_p(self.cand_table), context=_p(lens))
        ext.call("dsv41_reindex_table", a, _stream())
        # the compact table's rows are per decode row: row t reads table row t
        self._score(rows=rows, query=query, plane=plane, plan=None, itab=self.cand_table,
                    itab_stride=TOPK_BLOCKS, itab_len=TOPK_BLOCKS, entry_rows=BLOCK_ROWS,
                    owners=self.owners[0], bounds=lens, lstride=COMPACT, reindex=1,
                    reindex_chunks=COMPACT // CHUNK)
        return self.ilog[: rows * COMPACT].view(rows, COMPACT), lens, ids

    # ------------------------------------------------------------ selection
    def topk_of(self, vals, n, k, out, *, group=1, page_out=None, table=None, page=PLANE_ROWS, owners=None):
        a = abi.TopkArgs(rows=out.shape[0], k=k, vals=_p(vals), vstride=vals.stride(0), n=_p(n), group=group,
                         out=_p(out), page_out=_p(page_out), table=_p(table),
                         table_stride=0 if table is None else table.stride(0), page=page, owners=_p(owners))
        ext.call("dsv41_topk", a, _stream())

    def identity(self, *, rows, bounds, page_table, raw_out, page_out, owners=None):
        """Rows that see at most ``topk`` columns: every position in order, -1 padded, and its
        pool slot (SGLang's topk_transform_paged on such rows)."""
        owners = self.owners[0] if owners is None else owners
        self.topk_of(self.ilog, bounds, self.topk, raw_out, page_out=page_out, table=page_table, owners=owners)

    def select(self, *, kind, rows, per_req, ratio, query, plane, page_table, bounds, raw_out, page_out,
               candidates=None):
        """An index source's top-k of each row into raw_out / page_out [rows, topk] (positions
        ascending, -1 padded); a producer returns its candidate blocks."""
        if kind not in KINDS:
            raise RuntimeError(f"K2i: kind {kind!r} not in {KINDS}")
        if not (0 < rows <= MAX_ROWS and rows % per_req == 0):
            raise RuntimeError(f"K2i: {rows} rows, {per_req} a request")
        inputs = dict(rows=rows, per_req=per_req, query=query, plane=plane, page_table=page_table, bounds=bounds)
        owners = self.owners[per_req - 1]
        if kind == "reindex":
            compact, lens, ids = self.score_candidates(candidates=candidates, **inputs)
            pos = self.compact_pos[:rows]
            self.topk_of(compact, lens, self.topk, pos)
            a = abi.MapCompactArgs(rows=rows, topk=self.topk, block_rows=BLOCK_ROWS, page=PLANE_ROWS,
                                   compact=_p(pos), ids=_p(ids), ids_stride=ids.stride(0),
                                   page_table=_p(page_table), table_stride=page_table.stride(0),
                                   owners=_p(owners), raw_out=_p(raw_out), page_out=_p(page_out),
                                   out_stride=raw_out.stride(0))
            ext.call("dsv41_map_compact", a, _stream())
            return None
        logits = self.score(ratio=ratio, **inputs)
        published = None
        if kind == "producer":
            ids = self.cand_in[:rows]
            self.topk_of(logits, bounds, TOPK_BLOCKS, ids, group=BLOCK_ROWS)
            published = Candidates(ids)
        self.topk_of(logits, bounds, self.topk, raw_out, page_out=page_out, table=page_table, owners=owners)
        return published
