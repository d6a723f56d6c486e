from tileops.kernels.mamba.ssd_chunk_scan import SSDChunkScanFwdKernel

__all__ = ["SSDChunkScanFwdKernel"]
