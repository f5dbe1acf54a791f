"""Distributed layer: mesh, collectives, autograd mappings, executor, native NVLink comm."""
