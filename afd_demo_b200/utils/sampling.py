"""Token sampling: greedy, temperature, top-k, top-p (nucleus), repetition
penalty, and a stopping criterion. Same behaviour as the reference's
src/utils/sampling.py:13-196. Greedy decoding on a CUDA tensor runs the
framework's argmax kernel."""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F


def sample_next_token(logits: torch.Tensor, temperature: float = 1.0, top_k: int = 50,
                      top_p: float = 0.9, do_sample: bool = True,
                      generator: Optional[torch.Generator] = None) -> torch.Tensor:
    """logits [B, V] -> token ids [B, 1] (int64)."""
    if not do_sample:
        from .. import ops
        return ops.argmax(logits).view(-1, 1).long()
    if temperature != 1.0:
        logits = logits / temperature
    if top_k > 0:
        logits = top_k_filtering(logits, top_k)
    if top_p < 1.0:
        logits = top_p_filtering(logits, top_p)
    probs = F.softmax(logits.float(), dim=-1)
    return torch.multinomial(probs, num_samples=1, generator=generator)


def top_k_filtering(logits: torch.Tensor, top_k: int) -> torch.Tensor:
    top_k = min(top_k, logits.size(-1))
    kth = torch.topk(logits, top_k)[0][..., -1, None]
    return logits.masked_fill(logits < kth, float("-inf"))


def top_p_filtering(logits: torch.Tensor, top_p: float, min_tokens_to_keep: int = 1
                    ) -> torch.Tensor:
    sorted_logits, sorted_idx = torch.sort(logits, descending=True)
    cum = torch.cumsum(F.softmax(sorted_logits.float(), dim=-1), dim=-1)
    remove = cum > top_p
    remove[..., 1:] = remove[..., :-1].clone()
    remove[..., 0] = False
    remove[..., :min_tokens_to_keep] = False
    remove = remove.scatter(-1, sorted_idx, remove)
    return logits.masked_fill(remove, float("-inf"))


def repetition_penalty(logits: torch.Tensor, generated_ids: torch.Tensor,
                       penalty: float = 1.2) -> torch.Tensor:
    """Divide positive / multiply negative logits of already generated ids."""
    if penalty == 1.0:
        return logits
    logits = logits.clone()
    score = torch.gather(logits, 1, generated_ids)
    score = torch.where(score < 0, score * penalty, score / penalty)
    logits.scatter_(1, generated_ids, score)
    return logits


class StoppingCriteria:
    """Stop on max length or when every sequence has produced EOS."""

    def __init__(self, max_length: int, eos_token_id: Optional[int] = None,
                 pad_token_id: Optional[int] = None):
        self.max_length = max_length
        self.eos_token_id = eos_token_id
        self.pad_token_id = pad_token_id
        self._finished: Optional[torch.Tensor] = None

    def reset(self) -> None:
        self._finished = None

    def __call__(self, input_ids: torch.Tensor, next_tokens: torch.Tensor) -> bool:
        if input_ids.shape[1] >= self.max_length:
            return True
        if self.eos_token_id is None:
            return False
        done = next_tokens.view(-1) == self.eos_token_id
        self._finished = done if self._finished is None else (self._finished | done)
        return bool(self._finished.all())

    def get_finished_mask(self) -> Optional[torch.Tensor]:
        return self._finished

    def should_stop(self, input_ids: torch.Tensor, current_length: int) -> torch.Tensor:
        """Per-sequence stop mask [B] from the ids so far: every sequence at
        `max_length`, else the sequences whose last id is EOS (the reference's
        stateless check, src/utils/sampling.py:160-186)."""
        B = input_ids.shape[0]
        if current_length >= self.max_length:
            return torch.ones(B, dtype=torch.bool, device=input_ids.device)
        if self.eos_token_id is None:
            return torch.zeros(B, dtype=torch.bool, device=input_ids.device)
        return input_ids[:, -1] == self.eos_token_id

    def all_stopped(self, input_ids: torch.Tensor, current_length: int) -> bool:
        return bool(self.should_stop(input_ids, current_length).all())
