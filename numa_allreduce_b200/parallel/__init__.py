"""Schedules, CPU emulation, protocol selection and the communicator."""
