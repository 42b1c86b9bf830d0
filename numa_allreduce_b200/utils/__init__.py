"""Topology detection, environment configuration, logging and timing."""
