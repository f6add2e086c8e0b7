"""Polynomial flash attention (placeholder gate until the fused kernel lands)."""


def eligible(**bound):
    return False


def attention(**bound):
    raise NotImplementedError
