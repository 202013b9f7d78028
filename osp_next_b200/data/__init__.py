"""Data pipeline (reference: ospnext/data/*): datasets, stateful sampler, collator,
metadata stores, video IO and transforms."""
from .datasets import ospnext_datasets  # noqa: F401
from .dataloader import ospnext_samplers, ospnext_collators  # noqa: F401
