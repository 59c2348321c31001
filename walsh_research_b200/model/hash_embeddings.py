"""Hash embeddings (src/model/chassis.py:109-260): three shared tables of
`bucket_size` rows and a learned importance per (token, table) stand in for
the [vocab, n_embd] embedding.  The reference's mHCWalsh imports this class
from a module of this name (src/model/mhc.py:559-561); its chassis.py holds
the class itself.

Parameters, buffers and the universal-hashing constants are the reference's
(checkpoints load through load_state_dict).  On the device the class builds
the [vocab, n_embd] matrix it represents with walsh_hash_embed_rows, cached
with the model's other derived weights; lookups, the output projection and
the chunked cross entropy then use it."""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import _lib
from ..ops import require_cuda
from ._lib_call import call_hash_rows
from . import _prep


class HashEmbedding(nn.Module):
    def __init__(self, vocab_size: int, n_embd: int, bucket_size: int = 1021, num_tables: int = 3):
        super().__init__()
        self.bucket_size = bucket_size
        self.vocab_size = vocab_size
        self.n_embd = n_embd
        self.num_tables = num_tables
        self.emb_tables = nn.ModuleList([nn.Embedding(bucket_size, n_embd) for _ in range(num_tables)])
        self.importance = nn.Embedding(vocab_size, num_tables)
        for emb in self.emb_tables:
            nn.init.normal_(emb.weight, std=0.02 / math.sqrt(num_tables))
        nn.init.normal_(self.importance.weight, mean=1.0, std=0.01)
        # the reference's fixed hashing constants: a_t in [1, 1e5), b_t in [0, 1e5)
        # from NumPy's legacy RandomState(42), and the prime 1e9 + 7
        rng = np.random.RandomState(42)
        self.register_buffer("hash_a", torch.from_numpy(rng.randint(1, 100000, size=(num_tables, 1))).long())
        self.register_buffer("hash_b", torch.from_numpy(rng.randint(0, 100000, size=(num_tables, 1))).long())
        self.register_buffer("prime", torch.tensor(1000000007))
        ids = torch.arange(vocab_size)
        idx = ((ids * self.hash_a + self.hash_b) % self.prime) % bucket_size      # [num_tables, V]
        self.register_buffer("all_indices", idx.T.contiguous())                   # [V, num_tables]

    @property
    def scale(self) -> float:
        return math.sqrt(self.n_embd)

    def embedding_rows(self, start: int, end: int) -> torch.Tensor:
        """Rows start .. end - 1 of the represented embedding matrix, float32
        [end - start, n_embd], built on the device."""
        require_cuda(self.importance.weight)
        tables = torch.stack([e.weight.detach().float() for e in self.emb_tables]).contiguous()
        imp = self.importance.weight.detach().float().contiguous()
        ind = self.all_indices.to(torch.int64).contiguous()
        return call_hash_rows(tables, imp, ind, self.n_embd, self.scale, start, end)

    def weight_matrix(self) -> torch.Tensor:
        """The whole [vocab, n_embd] matrix (cached until a parameter changes)."""
        srcs = [e.weight for e in self.emb_tables] + [self.importance.weight, self.all_indices]
        return _prep.cached(self, "matrix", srcs, lambda: self.embedding_rows(0, self.vocab_size))

    def _get_chunk_embeddings(self, start: int, end: int) -> torch.Tensor:
        return self.embedding_rows(start, end)

    def _get_all_embeddings(self) -> torch.Tensor:
        return self.weight_matrix()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """[B, T] ids -> [B, T, n_embd] float32 embeddings."""
        return F.embedding(x, self.weight_matrix())

    def output_projection(self, hidden: torch.Tensor) -> torch.Tensor:
        """Logits [.., vocab] of hidden states [.., n_embd] against the matrix."""
        from .. import ops
        h = hidden.float().contiguous()
        flat = h.reshape(-1, self.n_embd)
        W = self.weight_matrix()
        if ops.split_eligible(flat, self.n_embd):
            y = ops.linear_split(flat, *ops.split_bf16(W))
        else:
            y = ops.linear(flat, W, None, out_dtype=torch.float32)
        return y.view(hidden.shape[:-1] + (self.vocab_size,))

    def chunked_cross_entropy(self, hidden: torch.Tensor, targets: torch.Tensor, chunk_size: int = 4096):
        """Mean cross entropy of the output projection against targets (the
        reference evaluates it in vocabulary chunks to bound memory; the value
        is the cross entropy of the full logits)."""
        logits = self.output_projection(hidden)
        return F.cross_entropy(logits.view(-1, self.vocab_size), targets.reshape(-1))

    def extra_repr(self) -> str:
        std_params = self.vocab_size * self.n_embd
        hash_params = self.bucket_size * self.n_embd * self.num_tables
        return f"vocab={self.vocab_size}, dim={self.n_embd}, bucket={self.bucket_size}, " \
               f"compression={std_params / hash_params:.1f}x"
