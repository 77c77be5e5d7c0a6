"""B200-native (sm_100a) fisheye Gaussian tracer with the GOFish interfaces.

The compute path is the C-ABI library libgofish_b200.so (include/gofish_b200.h)
built from gofish_b200/csrc; the Python modules mirror the reference's
threedgut_tracer entry points on top of it.
"""

__all__ = ["camera", "physical_tile_mask", "scene", "splat_raster"]
