"""Caller harnesses used to measure the operator inside whole training steps."""
