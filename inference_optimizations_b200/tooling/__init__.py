"""Operator tooling: scheduler trace, rooflines, accuracy gate, bounds checks (the reference's `tooling/`)."""
