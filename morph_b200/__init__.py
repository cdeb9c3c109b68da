"""morph_b200 — MORPH's optimizer-step hot path as hand-written sm_100a kernels.

Public drop-ins (same names and behaviour as the reference's interfaces):
  AdamW               torch.optim.AdamW as built at streamtrain/optimizer.py:40
  DynamicLossScale    streamtrain/precision.py:6-17, state resident on the GPU
  HybridMuonAdamW     streamtrain/optimizer.py:34-70 (Muon + AdamW); orthogonalize, partition
  morph_b200.disk     DeviceDiskState: DiskState.update arithmetic (streamtrain/disk.py:203-223)
                      on device-resident [w; m; v] planes, the row-sparse update, the
                      microbatch accumulation (accumulate_), the FP16 cast with export check
  morph_b200.disk_io  DiskState.update on the reference's state files (install, patch_class)
  morph_b200.export   the FP16 export writer (export_fp16)
  morph_b200.offload  row state in pinned host memory (OffloadedRowTable, ShardedRowTable)
  morph_b200.zero     one process per GPU: ZeroAdamW, ZeroHybridMuonAdamW
  morph_b200.precision pack_fp8 / unpack_fp8 (FP8 block transport)

All compute goes through the C-ABI library libmorph_b200.so (include/morph_b200.h);
importing a class that needs it raises ImportError when the library is missing.
"""
from .precision import DynamicLossScale, fp8_eligible
from .optim import AdamW
from .muon import HybridMuonAdamW, orthogonalize, partition

__all__ = ["AdamW", "DynamicLossScale", "HybridMuonAdamW", "fp8_eligible", "orthogonalize", "partition"]
