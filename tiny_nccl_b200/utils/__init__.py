"""Measurement helpers: device timing and clock sampling."""
from .clocks import ClockSampler, summarize

__all__ = ["ClockSampler", "summarize"]
