from .collator import WanDataCollator, LatentCollator
from .sampler import StatefulDistributedSampler

ospnext_samplers = {"stateful_distributed": StatefulDistributedSampler}
ospnext_collators = {"wan_t2v": WanDataCollator, "latent": LatentCollator}
