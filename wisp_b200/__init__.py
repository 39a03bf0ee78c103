"""wisp_b200 -- B200-native (sm_100a) MoE block forward behind WISP's C ABI.

* ``wisp_b200.lib``       -- ctypes binding of ``libwisp_b200.so`` (include/wisp_b200.h)
* ``wisp_b200.core``      -- mirror of the reference's ``_wisp_core`` module
* ``wisp_b200.moe``       -- device-resident MoE layers/stacks over the fused kernels
* ``wisp_b200.converter`` -- int4 quantiser, expert ``.bin`` format, seeded model writer
* ``wisp_b200.build``     -- nvcc build recipe (sm_100a)
"""

__version__ = "0.1.0"
