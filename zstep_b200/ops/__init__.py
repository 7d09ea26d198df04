"""Kernel-facing operations: thin wrappers over the sm_100a extension plus PyTorch
reference implementations of the same math (used by tests and the CPU plumbing model)."""
