"""Backpropagation through the recurrent spikes (``Drive.recurrent_gradients``)."""

from __future__ import annotations


def simulate(*args, **kwargs):
    raise NotImplementedError("gradients through the recurrent spikes are not built yet")
