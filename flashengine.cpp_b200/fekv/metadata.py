"""Per-step paged-KV metadata: the host assembly the reference performs in
``CudaModel::prepare`` (Cambridgebit/FlashEngine.cpp src/cuda_model.cpp:131-142).

From each scheduled sequence's block table (``Sequence::blocks``,
include/fe/scheduler.hpp:15), its first position written this step and its row
count, build:

* ``slots``  int64 [rows]: ``blocks[pos // page] * page + pos % page`` for every
  new token (the append's slot mapping, :136);
* ``qo``     int32 [batch+1]: query-row prefix sums;
* ``kv``     int32 [batch+1]: page-count prefix sums;
* ``pages``  int32: each sequence's first ceil(length/page) block ids;
* ``last``   int32 [batch]: ``(length-1) % page + 1``.

Graph padding (:138): padded entries get ``rows`` rows with ``slot = -1``, one
page (the dummy page ``num_blocks``) and ``last = rows``.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class StepMetadata:
    slots: np.ndarray
    positions: np.ndarray
    qo: np.ndarray
    kv: np.ndarray
    pages: np.ndarray
    last: np.ndarray

    @property
    def batch(self) -> int:
        return int(self.kv.shape[0] - 1)

    @property
    def rows(self) -> int:
        return int(self.qo[-1])

    def lengths(self, page: int) -> np.ndarray:
        return (self.kv[1:] - self.kv[:-1] - 1).astype(np.int64) * page + self.last


def build_step_metadata(block_tables, starts, rows, page, pad_to=None, pad_rows=1,
                        dummy_page=None) -> StepMetadata:
    """block_tables: list of int arrays; starts[b]: first position written
    this step; rows[b]: tokens written (= query rows) this step."""
    slots, positions, pages = [], [], []
    qo, kv, last = [0], [0], []
    for blocks, start, n in zip(block_tables, starts, rows):
        blocks = np.asarray(blocks, dtype=np.int64)
        start, n = int(start), int(n)
        length = start + n
        pos = np.arange(start, length, dtype=np.int64)
        if pos.size and int(pos[-1] // page) >= blocks.size:
            raise ValueError("block table does not cover the write slots")
        slots.append(blocks[pos // page] * page + pos % page)
        positions.append(pos)
        qo.append(qo[-1] + n)
        npages = -(-length // page)
        if npages > blocks.size:
            raise ValueError("block table does not cover the context")
        pages.append(blocks[:npages])
        kv.append(kv[-1] + npages)
        last.append((length - 1) % page + 1)
    if pad_to is not None:
        if dummy_page is None:
            raise ValueError("graph padding needs the dummy page id")
        for _ in range(len(block_tables), int(pad_to)):
            slots.append(np.full(pad_rows, -1, dtype=np.int64))
            positions.append(np.arange(pad_rows, dtype=np.int64))
            qo.append(qo[-1] + pad_rows)
            pages.append(np.array([dummy_page], dtype=np.int64))
            kv.append(kv[-1] + 1)
            last.append(pad_rows)
    cat = lambda xs, dt: np.concatenate(xs).astype(dt) if xs else np.zeros(0, dt)  # noqa: E731
    return StepMetadata(slots=cat(slots, np.int64), positions=cat(positions, np.int64),
                        qo=np.asarray(qo, np.int32), kv=np.asarray(kv, np.int32),
                        pages=cat(pages, np.int32), last=np.asarray(last, np.int32))


def draft_block_metadata(blocks, start, rows, page) -> StepMetadata:
    """A DFlash draft block of one sequence as paged metadata: `rows` new
    positions [start, start + rows) that attend, with the full (non-causal)
    mask, to every position < start + rows. This is the read_ / valid_ of the
    reference's ReferenceBlockDraft::propose (src/block_draft.cpp:50-53), which
    gathers max_model_len slots and masks those at or beyond `valid`; here the
    same keys come from the block table, so the attention reads only them."""
    return build_step_metadata([np.asarray(blocks, np.int64)], [int(start)], [int(rows)], page)

