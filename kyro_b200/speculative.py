"""The verify half of the reference's SpeculativeDecoder, batched.

Mirrors ``SpeculativeDecoder::verify_drafts`` (src/speculative.rs:286-339):
given the target model's logits over the drafted positions and the draft
tokens, decide how many drafts to accept and which token to emit next.
The reference compares argmaxes (greedy); ``ACCEPT_GREEDY_REF`` reproduces
that rule exactly (no bonus token, k == 0 emits one argmax),
``ACCEPT_GREEDY`` adds the bonus token, and ``ACCEPT_STOCHASTIC`` is
rejection sampling with seeded Philox uniforms.  All modes run in the
sm_100a sampler kernels (kyro_spec_accept).
"""
from __future__ import annotations

from typing import List, Optional

import torch

from .verify import (ACCEPT_GREEDY, ACCEPT_GREEDY_REF, ACCEPT_STOCHASTIC, Context, sample_tokens,
                     spec_accept)


class DraftStrategy:
    """Names of the reference's draft strategies (src/speculative.rs:139-146)."""
    DRAFT_MODEL = "DraftModel"
    NGRAM = "Ngram"
    PARALLEL = "Parallel"


class SpeculativeVerifier:
    def __init__(self, lookahead: int, mode: int = ACCEPT_GREEDY_REF, temperature: float = 1.0,
                 seed: int = 0, ctx: Optional[Context] = None):
        self.lookahead = lookahead
        self.mode = mode
        self.temperature = temperature
        self.seed = seed
        self.step_counter = 0
        self._ctx = ctx

    def _context(self, device) -> Context:
        if self._ctx is None or self._ctx.device != device:
            self._ctx = Context(device.index)
        return self._ctx

    def verify_drafts(self, target_logits: torch.Tensor, draft_tokens: torch.Tensor,
                      draft_logits: Optional[torch.Tensor] = None, step: Optional[int] = None,
                      seq_offset: int = 0):
        """target_logits [B, k+1, V] (or [k+1, V] for one sequence), draft
        tokens [B, k].  Returns (accept_len, tokens, num_tokens)."""
        single = target_logits.dim() == 2
        tl = target_logits.unsqueeze(0) if single else target_logits
        dt = draft_tokens.reshape(tl.shape[0], tl.shape[1] - 1).to(torch.int32).contiguous()
        dl = None
        if draft_logits is not None:
            dl = (draft_logits.unsqueeze(0) if single else draft_logits).float().contiguous()
        st = self.step_counter if step is None else step
        if step is None:
            self.step_counter += 1
        ctx = self._context(tl.device)
        acc, toks, num, _ = spec_accept(ctx, tl.float().contiguous(), dl, dt, self.mode,
                                        self.temperature, self.seed, st, seq_offset)
        return acc, toks, num

    @staticmethod
    def to_lists(tokens: torch.Tensor, num_tokens: torch.Tensor) -> List[List[int]]:
        """Per-sequence emitted tokens, as the reference's Vec<u32>."""
        t = tokens.cpu().tolist()
        n = num_tokens.cpu().tolist()
        return [row[:c] for row, c in zip(t, n)]

    def sample_drafts(self, draft_logits: torch.Tensor, temperature: Optional[float] = None,
                      step: int = 0, seq_offset: int = 0):
        """On-device draft sampling from softmax(draft_logits / T), Philox
        stream 0; T <= 0 is argmax as in the reference draft loop
        (src/speculative.rs:232-236)."""
        ctx = self._context(draft_logits.device)
        T = self.temperature if temperature is None else temperature
        return sample_tokens(ctx, draft_logits.float().contiguous(), T, self.seed, step,
                             seq_offset)
