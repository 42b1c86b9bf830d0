"""Native op wrappers: allreduce emulation group, fused allreduce + RMSNorm."""
