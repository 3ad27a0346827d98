"""RCO: budget manifold (host, float64) and the exact MCKP decode on the GPU."""
