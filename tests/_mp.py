"""Results of spawned test ranks cross the queue as numpy arrays: torch tensors
would be shared through file descriptors that vanish when the child exits
before the parent has unpickled them."""
import numpy as np
import torch


def to_host(obj):
    """Tensors (anywhere in tuples, lists, dicts) -> numpy arrays, recursively."""
    if torch.is_tensor(obj):
        t = obj.detach().cpu()
        if t.dtype == torch.bfloat16:
            return ("bf16", t.view(torch.int16).numpy().copy())
        return t.numpy().copy()
    if isinstance(obj, tuple):
        return tuple(to_host(x) for x in obj)
    if isinstance(obj, list):
        return [to_host(x) for x in obj]
    if isinstance(obj, dict):
        return {k: to_host(v) for k, v in obj.items()}
    return obj


def from_host(obj):
    """Inverse of to_host."""
    if isinstance(obj, np.ndarray):
        return torch.from_numpy(obj)
    if isinstance(obj, tuple):
        if len(obj) == 2 and obj[0] == "bf16" and isinstance(obj[1], np.ndarray):
            return torch.from_numpy(obj[1]).view(torch.bfloat16)
        return tuple(from_host(x) for x in obj)
    if isinstance(obj, list):
        return [from_host(x) for x in obj]
    if isinstance(obj, dict):
        return {k: from_host(v) for k, v in obj.items()}
    return obj
