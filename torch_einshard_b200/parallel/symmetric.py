"""Peer-mapped symmetric buffers and native communicators (filled in with the comm kernels)."""


def activate(mesh=None):
    return False
