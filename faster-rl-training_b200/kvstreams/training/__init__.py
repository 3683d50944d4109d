from .logprobs import token_logprobs
from .mismatch import MismatchReport, measure_mismatch, mismatch_report
from .replay import (
    Batch,
    TrainSequence,
    build_sequences,
    collate,
    full_context_sequence,
    kvstream_sequence,
    window_sequences,
)

__all__ = [
    "Batch",
    "MismatchReport",
    "TrainSequence",
    "build_sequences",
    "collate",
    "full_context_sequence",
    "kvstream_sequence",
    "measure_mismatch",
    "mismatch_report",
    "token_logprobs",
    "window_sequences",
]
