"""Tokenized documents in a memory-mapped Arrow IPC file (the host input path).

The file layout is Quail's TokenStore (quail/execution/tokens.py:180-359):
one IPC file of record batches with a ``__quail_token_ids`` column
(large_list of an integer token type) and a ``__quail_token_count`` int64
column, schema metadata ``quail.kind = token_store``. A store Quail wrote
opens here and one written here opens in Quail.

``TokenStore[i]`` is a zero-copy numpy view of document i's tokens into the
mapped file, so a filter over millions of rows materialises only the rows
each chunk packs; ``lengths`` reads the count column without touching the
tokens. The loop's packer concatenates these views into the chunk's
``input_ids`` (one pinned upload per chunk array).
"""

import bisect
from collections.abc import Sequence

import numpy as np
import pyarrow as pa

TOKEN_COLUMN = "__quail_token_ids"
COUNT_COLUMN = "__quail_token_count"


class TokenStore(Sequence):
    """Random access to the documents of one token store file."""

    def __init__(self, path):
        self.path = str(path)
        self._source = pa.memory_map(self.path, "r")
        reader = pa.ipc.open_file(self._source)
        self._offsets, self._values, self._counts, self._ends = [], [], [], []
        total = 0
        for b in range(reader.num_record_batches):
            batch = reader.get_batch(b)
            tokens = batch.column(batch.schema.get_field_index(TOKEN_COLUMN))
            counts = batch.column(batch.schema.get_field_index(COUNT_COLUMN))
            self._offsets.append(tokens.offsets.to_numpy(zero_copy_only=True))
            self._values.append(tokens.values.to_numpy(zero_copy_only=True))
            self._counts.append(counts.to_numpy(zero_copy_only=True))
            total += len(batch)
            self._ends.append(total)
        self.lengths = _Lengths(self)

    def __len__(self):
        return self._ends[-1] if self._ends else 0

    def _locate(self, index):
        if index < 0:
            index += len(self)
        if not 0 <= index < len(self):
            raise IndexError(index)
        b = bisect.bisect_right(self._ends, index)
        return b, index - (self._ends[b - 1] if b else 0)

    def __getitem__(self, index):
        if isinstance(index, slice):
            return [self[i] for i in range(*index.indices(len(self)))]
        b, local = self._locate(index)
        off = self._offsets[b]
        return self._values[b][int(off[local]):int(off[local + 1])]

    def close(self):
        self._source.close()


class _Lengths(Sequence):
    """Document lengths from the count column (no token reads)."""

    def __init__(self, store):
        self._store = store

    def __len__(self):
        return len(self._store)

    def __getitem__(self, index):
        if isinstance(index, slice):
            return [self[i] for i in range(*index.indices(len(self)))]
        b, local = self._store._locate(index)
        return int(self._store._counts[b][local])


def write_token_store(path, documents, token_type=pa.int32(), batch_rows=65536):
    """Write token sequences as a token store file; returns it opened."""
    list_type = pa.large_list(token_type)
    schema = pa.schema([pa.field(TOKEN_COLUMN, list_type, nullable=False),
                        pa.field(COUNT_COLUMN, pa.int64(), nullable=False)],
                       metadata={b"quail.kind": b"token_store"})
    with pa.OSFile(str(path), "wb") as sink, pa.ipc.new_file(sink, schema) as writer:
        for lo in range(0, len(documents), batch_rows):
            docs = [np.asarray(d) for d in documents[lo:lo + batch_rows]]
            tokens = pa.array(docs, type=list_type)
            counts = pa.array([len(d) for d in docs], type=pa.int64())
            writer.write_batch(pa.RecordBatch.from_arrays([tokens, counts], schema=schema))
    return TokenStore(path)
