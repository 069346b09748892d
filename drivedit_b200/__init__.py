import torch  # noqa: F401  (loads libc10 before the extension)
