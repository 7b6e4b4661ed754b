import torch


def rel_err(x, ref):
    """Relative L2 error of x against ref (the reference test harness's metric)."""
    x = x.float()
    ref = ref.float()
    den = ref.norm().item()
    return (x - ref).norm().item() / (den if den > 0 else 1.0)
