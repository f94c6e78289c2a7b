"""mamba4_b200: the Mamba 4 FlashMamba hot path, native on B200 (sm_100a).

Operators (reference `lm/kernels` surface):
  memory:      selective_memory_fused, selective_gaussian_memory,
               selective_decode, SelectiveState, SelectiveResult,
               selective_initial_state, spd_solve
  flashmamba:  mamba3_fused, mamba3_flash, mamba3_flash_heads, angle_rates,
               mamba3_step, mamba3_step_cache, Mamba3StepCache
Compute runs in the in-tree CUDA library `libmamba4_b200.so` (C ABI in
include/mamba4_b200.h); importing the package does not need a GPU.
"""

from .memory import (  # noqa: F401
    SelectiveResult,
    SelectiveState,
    selective_decode,
    selective_gaussian_memory,
    selective_initial_state,
    selective_memory_fused,
    spd_solve,
)
from .flashmamba import (  # noqa: F401
    Mamba3StepCache,
    angle_rates,
    mamba3_flash,
    mamba3_flash_heads,
    mamba3_fused,
    mamba3_step,
    mamba3_step_cache,
)

__version__ = "0.1"
