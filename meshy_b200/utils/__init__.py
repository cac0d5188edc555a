"""Utilities: samples, timers, metrics, HF snapshot resolution."""
