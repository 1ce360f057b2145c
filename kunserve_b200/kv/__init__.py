from .layout import KVLayout, fusion_id, split_fusion_id
from .block_manager import BlockManager, NoFreeBlocksError, BlockLocation
