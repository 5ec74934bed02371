"""Python access to the B200 Sana denoiser library (``lib/libsana_cuda.so``, C ABI of
``include/sana_cuda.h``). The product is the C ABI; this package is a thin ctypes layer
used by tests, ``bench.py`` and ``__graft_entry__``. It never falls back to a CPU path:
if the shared library is missing or no CUDA device is present, calls fail loudly."""
from .capi import (  # noqa: F401
    SANA_LAYOUT_REFERENCE,
    SANA_LAYOUT_TORCH,
    SANA_MODE_BF16,
    SANA_MODE_F32,
    SanaCuda,
    SanaError,
    gemm_counts,
    gguf_index,
    lib_path,
    load_library,
    prompt_pair_assemble,
    randn_torch_cpu,
    scheduler_config,
    scheduler_schedule,
    scheduler_schedule_config,
    select_rows_first_and_last,
)
