"""quest: Quest top-K page selection (exports of src/quest/__init__.py:23-34),
computed by the CUDA library ``libhelix_kv.so``."""
from .reference import compute_page_stats, page_upper_bound, selected_attention, topk_pages_with_sinks

__all__ = [
    "compute_page_stats",
    "page_upper_bound",
    "topk_pages_with_sinks",
    "selected_attention",
]
