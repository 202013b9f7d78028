"""Measurement programs behind the committed profile summaries (per-kernel timing against
the measured peaks, the fused SSP exchange and FSDP collectives against their NVLink
rooflines, exposed communication of a training step).  Run as ``python -m benchmarks.<name>``
(``torchrun ... -m benchmarks.<name>`` for the multi-GPU ones) from the repository root."""
