"""Load the product's ctypes binding (the package directory name is not a
Python identifier, so it is loaded by path)."""
import importlib.util
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "disk-qwen35ba3b_b200")


def ds4f_cuda():
    spec = importlib.util.spec_from_file_location(
        "ds4f_cuda", os.path.join(PKG, "ds4f_cuda.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def gpu_available():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
