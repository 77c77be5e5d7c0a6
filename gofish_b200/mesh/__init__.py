"""Mesh opacity query of the B200 tracer: the matched camera-min opacity
field and the bisection of Marching-Tetrahedra crossing edges.

Module layout follows the reference's ``gofish.mesh`` package:
``raster`` (the native SplatRaster methods), ``field``, ``bisection``,
``shape``, ``sites`` and ``cameras``.  Tetrahedralization, marching
tetrahedra and the mesh filters are not part of this package.
"""

from .raster import SplatRaster

__all__ = ["SplatRaster"]
