"""B200-native (sm_100a) DCNv2 -- modulated deformable convolution, forward and backward.

Drop-in for the reference's ``Conv2d._C`` ops and ``dcn_v2_mm`` modules:

    from dcnv2_b200 import _C                     # was: from Conv2d import _C
    from dcnv2_b200 import DCN, DCNv2, dcn_v2_conv  # was: from dcn_v2_mm import ...
"""
from . import _C  # noqa: F401  (loads libdcn_b200.so; raises ImportError if it is not built)
from ._lib import version  # noqa: F401
from .modules import DCN, DCNv2, _DCNv2, dcn_v2_conv, dcn_v2_conv_om  # noqa: F401

__all__ = ["_C", "DCN", "DCNv2", "dcn_v2_conv", "dcn_v2_conv_om", "version"]
