from .spans import Span, in_spans, merge_spans, positions_to_spans, span_length

__all__ = ["Span", "in_spans", "merge_spans", "positions_to_spans", "span_length"]
