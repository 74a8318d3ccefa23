"""dion_b200: Blackwell-native (sm_100a) distributed orthonormalizing optimizers.

Muon, Dion, Dion2, AdaDion and AdaDionV2 (plus the research variants SDion,
GSDion, AGDion and QCDion) with torch.optim-style constructors, backed by
hand-written tcgen05/TMA kernels and NVLink collectives.
"""

import torch as _torch  # noqa: F401  (loads libc10 / libtorch before the native extension ``dion_b200._C``)

__version__ = "0.1.0"
