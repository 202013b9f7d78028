from .t2v import T2VInferencePipeline

pipelines = {"t2v": T2VInferencePipeline}
pipeline = pipelines
