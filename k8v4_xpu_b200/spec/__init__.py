"""Speculative decoding: the MTP drafter and its acceptance logging."""
