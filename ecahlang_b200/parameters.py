"""Request sampling parameters and their normalisation.

Mirrors ecahLang's OpenAI request form (ecahlang/parameters.py:4-12) and the
normalisation its stream() applies before queueing a request
(ecahlang/main.py:642-645): temperature is clamped to >= 1e-5 (so T = 0 is
sampled at T = 1e-5, not taken greedily), top_k = 0 means the whole
vocabulary, top_p = 0 means 1.0, repetition_penalty is clamped to >= 1e-5.

frequency_penalty and presence_penalty are additions (OpenAI-style additive
penalties, default 0 = off); the reference has no such fields.
"""
from __future__ import annotations

from dataclasses import dataclass

from pydantic import BaseModel


class Parameters(BaseModel):
    """The sampling knobs of a completion request (the reference's fields,
    plus the two optional additive penalties)."""
    model: str = "model"
    temperature: float = 1.0
    top_p: float = 0
    top_k: int = 0
    max_tokens: int = 256
    repetition_penalty: float = 1.0
    ignore_eos: bool = False
    stream: bool = False
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0


@dataclass(frozen=True)
class RowParams:
    """One request's normalised per-step sampling parameters."""
    temperature: float
    top_k: int
    top_p: float
    repetition_penalty: float
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0


def normalize(form: Parameters, vocab_size: int) -> RowParams:
    """ecahlang/main.py:642-645."""
    return RowParams(
        temperature=max(1e-5, form.temperature),
        top_k=vocab_size if form.top_k == 0 else form.top_k,
        top_p=1.0 if form.top_p == 0 else form.top_p,
        repetition_penalty=max(1e-5, form.repetition_penalty),
        frequency_penalty=form.frequency_penalty,
        presence_penalty=form.presence_penalty,
    )
