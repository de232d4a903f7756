"""Namespace for the B200-native sf hot path: ``superfloat.python_b200``."""
