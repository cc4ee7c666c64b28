"""Runnable examples (``python -m flodl_b200.examples.<name>``)."""
