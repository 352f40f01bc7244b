"""Ordered, bounded parallel tokenization for dataset preparation (reference
tnlm/data_preparation.py:17-127).

Documents are grouped into batches of at most ``batch_bytes`` UTF-8 bytes (128 documents at most; a
larger document forms a batch alone) and tokenized by a process pool (GPT-2 BPE loaded once per
worker).  Results come back strictly in input order, with at most ``2 * workers`` batches queued,
so the output bytes never depend on the worker count.  ``workers == 1`` runs in-process.
"""
from __future__ import annotations

import hashlib
import multiprocessing
from collections import deque
from concurrent.futures import ProcessPoolExecutor

import numpy as np

from .token_format import TOKEN_DTYPE

GPT2_VOCAB = 50257
_WORKER_TOKENIZER = None


def _init_worker(tokenizer):
    global _WORKER_TOKENIZER
    if tokenizer is None:
        import tiktoken
        tokenizer = tiktoken.get_encoding("gpt2")
    _WORKER_TOKENIZER = tokenizer


def _normalise(text: str) -> str:
    return text.replace("\r\n", "\n").replace("\r", "\n")


def encode_batch(batch, tokenizer=None):
    """[(doc_id, text, ...extra)] -> [(doc_id, processed_sha256, int64 token array, ...extra)]."""
    tok = _WORKER_TOKENIZER if tokenizer is None else tokenizer
    out = []
    for doc_id, text, *extra in batch:
        processed = _normalise(text)
        ids = np.asarray(tok.encode(processed, allowed_special=set(), disallowed_special=()), dtype="<i8")
        if len(ids) and (ids.min() < 0 or ids.max() >= GPT2_VOCAB):
            raise ValueError("tokens must belong to the real GPT2 vocabulary")
        out.append((doc_id, hashlib.sha256(processed.encode("utf-8")).hexdigest(), ids, *extra))
    return out


def batches(rows, byte_limit):
    batch, size = [], 0
    for row in rows:
        n = len(row[1].encode("utf-8"))
        if batch and (size + n > byte_limit or len(batch) >= 128):
            yield batch
            batch, size = [], 0
        batch.append(row)
        size += n
    if batch:
        yield batch


def ordered_tokenization(rows, *, tokenizer, workers, batch_bytes):
    """Yield ``encode_batch`` results for ``rows`` in input order.

    ``tokenizer`` None means GPT-2 (each worker loads its own); an injected tokenizer must pickle."""
    if type(workers) is not int or workers < 1:
        raise ValueError("workers must be a positive integer")
    if type(batch_bytes) is not int or batch_bytes < 1:
        raise ValueError("tokenization batch bytes must be a positive integer")
    it = iter(batches(rows, batch_bytes))
    if workers == 1:
        if tokenizer is None:
            _init_worker(None)
        for batch in it:
            yield from encode_batch(batch, tokenizer)
        return
    ctx = multiprocessing.get_context("fork")
    with ProcessPoolExecutor(workers, mp_context=ctx, initializer=_init_worker, initargs=(tokenizer,)) as pool:
        pending = deque()
        for batch in it:
            pending.append(pool.submit(encode_batch, batch))
            if len(pending) >= 2 * workers:
                yield from pending.popleft().result()
        while pending:
            yield from pending.popleft().result()


def token_array(ids: np.ndarray) -> np.ndarray:
    return ids.astype(TOKEN_DTYPE)
