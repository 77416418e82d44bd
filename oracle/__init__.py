"""Test infrastructure: CPU oracle and reference-build recipe. Not shipped."""
