from tileops.ops.mamba.ssd_chunk_scan import SSDChunkScanFwdOp

__all__ = ["SSDChunkScanFwdOp"]
