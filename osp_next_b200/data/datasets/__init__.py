from .t2v_dataset import T2VRandomDataset, T2VRandomLatentDataset, WanT2VDataset

ospnext_datasets = {
    "wan_t2v": WanT2VDataset,
    "t2v_random": T2VRandomDataset,
    "t2v_random_latent": T2VRandomLatentDataset,
}
