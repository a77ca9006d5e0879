"""Device guard for custom launches (mirror of utils/cuda.py:10-22)."""

from functools import wraps

import torch


def on_tensor_device(function):
    """Run custom launches on the tensor's device, preserving its current stream."""
    @wraps(function)
    def wrapped(*args, **kwargs):
        tensor = next((value for value in (*args, *kwargs.values())
                       if isinstance(value, torch.Tensor)), None)
        if tensor is None or not tensor.is_cuda:
            return function(*args, **kwargs)
        if tensor.device.index == torch.cuda.current_device():
            return function(*args, **kwargs)
        with torch.cuda.device(tensor.device):
            return function(*args, **kwargs)
    return wrapped
