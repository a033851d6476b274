"""gs_b200: B200-native (sm_100a) differentiable tiled Gaussian-splat renderer.

Drop-in mirror of jax-gs's renderer package: the module layout, function
names, signatures and constants follow jax_gs.core / jax_gs.renderer /
jax_gs.training, over torch CUDA tensors, with every stage running in the
hand-written kernels of libgsb200.so (include/gsb200.h).
"""
from gs_b200.core.camera import Camera
from gs_b200.core.gaussians import Gaussians
from gs_b200.renderer.renderer import render

__all__ = ["Camera", "Gaussians", "render"]
