"""Pattern lowerings for dense contractions (filled in by the tcgen05 kernels)."""


def try_lower(graph, node, kmeta, prefix, options):
    return None
