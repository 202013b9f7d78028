from .flow_matching import FlowMatchingScheduler

schedulers = {"flow_matching": FlowMatchingScheduler}
