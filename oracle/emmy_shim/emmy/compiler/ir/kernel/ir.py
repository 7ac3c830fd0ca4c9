from emmy.compiler._model import (  # noqa: F401
    CpAsyncCommit, CpAsyncCopy, CpAsyncWait, KernelOp, LdmatrixLoad, MmaSyncPtx, RegFragment, RegStore,
    Smem, Sync, Tile, TreeHalve, WarpShuffle,
)
