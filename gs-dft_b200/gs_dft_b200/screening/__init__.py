"""Significant-overlap pair screening on the device."""
from .pairs import count_significant, neighbor_pairs, pair_weight, stripe_pairs

__all__ = ["neighbor_pairs", "count_significant", "pair_weight", "stripe_pairs"]
