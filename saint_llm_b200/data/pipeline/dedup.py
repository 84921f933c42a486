"""Exact (SHA1 fingerprint) and near-duplicate (MinHash signature) dedup stages.

MinHash signatures come from the native extension: one 64-bit hash per character
5-shingle and ``n_perm`` universal permutations ``(a x + b) mod (2^61 - 1)`` (Broder),
batched over documents.  Two documents are duplicates when their full signatures match,
the dedup rule of ``saint_llm_data/pipeline/dedup.py:90-120``.
"""

from __future__ import annotations

import hashlib
from collections.abc import Sequence
from dataclasses import dataclass, field

import numpy as np
import torch

from saint_llm_b200.data.pipeline.stage import Document


def minhash_signatures(texts: Sequence[str], *, n_perm: int = 128, shingle: int = 5, seed: int = 1) -> torch.Tensor:
    """(len(texts), n_perm) int64 signatures; an empty text gives all zeros."""
    from saint_llm_b200.ops.backend import ext

    cps = [np.frombuffer(t.encode("utf-32-le"), dtype=np.int32) for t in texts]
    offs = np.zeros(len(cps) + 1, dtype=np.int64)
    np.cumsum([c.size for c in cps], out=offs[1:])
    flat = torch.from_numpy(np.concatenate(cps) if cps else np.zeros(0, np.int32))
    return ext().minhash_signatures(flat, torch.from_numpy(offs), n_perm, shingle, seed)


def minhash_signature(text: str, *, n_perm: int = 128) -> tuple[int, ...]:
    return tuple(int(v) for v in minhash_signatures([text], n_perm=n_perm)[0])


@dataclass
class FingerprintDedup:
    name: str = "fingerprint_dedup"
    _seen: set[bytes] = field(default_factory=set)

    def __call__(self, doc: Document) -> Document | None:
        text = doc.get("text", "")
        if not text:
            return doc
        fp = hashlib.sha1(text.encode("utf-8")).digest()
        if fp in self._seen:
            return None
        self._seen.add(fp)
        return doc

    def __len__(self) -> int:
        return len(self._seen)

    def reset(self) -> None:
        self._seen.clear()


@dataclass
class MinHashDedup:
    n_perm: int = 128
    name: str = "minhash_dedup"
    _seen: set[bytes] = field(default_factory=set)

    def __call__(self, doc: Document) -> Document | None:
        text = doc.get("text", "")
        if not text:
            return doc
        key = minhash_signatures([text], n_perm=self.n_perm).numpy().tobytes()
        if key in self._seen:
            return None
        self._seen.add(key)
        return doc

    def filter_batch(self, docs: Sequence[Document]) -> list[Document]:
        """Vectorised form: one native call signs the whole batch."""
        sigs = minhash_signatures([d.get("text", "") for d in docs], n_perm=self.n_perm).numpy()
        out = []
        for d, s in zip(docs, sigs, strict=True):
            if not d.get("text", ""):
                out.append(d)
                continue
            key = s.tobytes()
            if key not in self._seen:
                self._seen.add(key)
                out.append(d)
        return out

    def __len__(self) -> int:
        return len(self._seen)

    def reset(self) -> None:
        self._seen.clear()
