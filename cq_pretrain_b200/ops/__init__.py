"""Ops layer: each op has a plain-PyTorch oracle (``reference``) and an sm_100a kernel path."""
