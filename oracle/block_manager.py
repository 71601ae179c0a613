"""CPU oracle for the paged block bookkeeping -- TEST INFRASTRUCTURE ONLY.

The checker for the device-side block pool (csrc/block_pool.cu); only
``tests/`` import it.  Pure Python restating, step for step, the reference's
host code:

* ``BlockManager``        -- core/block_manager.py:19-68: a LIFO free list
                             initialised to ``list(range(num_blocks))``;
                             ``allocate`` pops ``num_blocks`` ids off the end
                             (:36-37) and appends them to the sequence's list
                             (:39-42), or returns INSUFFICIENT_SPACE without
                             change (:32-33); ``release_blocks`` pushes the
                             sequence's ids back in list order (:52-55) or
                             returns FAILURE for an unknown sequence (:49-50).
* ``padded_block_table``  -- transformer/model.py:126-152: ``num_blocks_per_seq``
                             from the dict in the step's sequence order and a
                             zero-padded int32 [S, max_blocks] table.
* ``step_metadata``       -- core/model_runner.py:66-107: per-sequence q_len /
                             kv_len / offsets and per-token positions and
                             sequence ids, prefill sequences first; the decode
                             rows use the runner's position ``len(token_ids)``
                             and kv_len ``len(token_ids) + 1`` (one past the
                             last token) unless ``fixed_positions`` is set, in
                             which case the decode token sits at
                             ``len(token_ids) - 1`` and kv_len is
                             ``len(token_ids)``.

Parity status: pinned.  tests/golden/block_trace.npz records the reference's
own Scheduler and BlockManager over a seeded request trace;
tests/test_block_pool_cpu.py replays it through this module.
"""
from __future__ import annotations

SUCCESS, INSUFFICIENT_SPACE, FAILURE = 0, 1, 2


class BlockManager:
    """core/block_manager.py:19-68 (statuses as ints: 0 success, 1 insufficient space, 2 failure)."""

    def __init__(self, num_blocks: int, block_size: int):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.st = list(range(num_blocks))
        self.block_table: dict[int, list[int]] = {}

    def allocate(self, seq_id: int, num_blocks: int) -> tuple[int, list[int]]:
        if len(self.st) < num_blocks:
            return INSUFFICIENT_SPACE, []
        ids = [self.st.pop() for _ in range(num_blocks)]
        self.block_table.setdefault(seq_id, []).extend(ids)
        return SUCCESS, ids

    def release_blocks(self, seq_id: int) -> int:
        if seq_id not in self.block_table:
            return FAILURE
        self.st.extend(self.block_table.pop(seq_id))
        return SUCCESS

    def num_free_blocks(self) -> int:
        return len(self.st)

    def can_allocate(self, num_blocks: int) -> bool:
        return len(self.st) >= num_blocks


def padded_block_table(block_table: dict, sequence_ids) -> tuple[list[list[int]], list[int]]:
    """transformer/model.py:126-152 (lists instead of tensors)."""
    nblk = [len(block_table[int(s)]) for s in sequence_ids]
    width = max(nblk) if nblk else 0
    rows = []
    for s in sequence_ids:
        ids = block_table[int(s)]
        rows.append(list(ids) + [0] * (width - len(ids)))
    return rows, nblk


def step_metadata(prefill: list[tuple[int, int, int]], decode: list[tuple[int, int, int]],
                  fixed_positions: bool = False) -> dict:
    """core/model_runner.py:66-107.

    ``prefill`` / ``decode``: (seq_id, len(prompt_token_ids), len(token_ids))
    per scheduled sequence, in the scheduler's order.
    """
    sequence_id, length, offset, position_ids, pos_seq_id, kv_len = [], [], [], [], [], []
    cnt = 0
    for sid, n_prompt, n_tok in prefill:
        sequence_id.append(sid)
        length.append(n_prompt)
        offset.append(cnt)
        cnt += n_prompt
        pos_seq_id.extend([sid] * n_prompt)
        position_ids.extend(range(n_tok))
        kv_len.append(n_prompt)
    for sid, _, n_tok in decode:
        sequence_id.append(sid)
        length.append(1)
        offset.append(cnt)
        cnt += 1
        pos_seq_id.append(sid)
        position_ids.append(n_tok - 1 if fixed_positions else n_tok)
        kv_len.append(n_tok if fixed_positions else n_tok + 1)
    return dict(sequence_id=sequence_id, q_len=length, offset=offset, position_ids=position_ids,
                pos_seq_id=pos_seq_id, kv_len=kv_len)
