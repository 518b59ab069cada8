"""DGL DataLoader wrapper (GIDS.py:143-488), imported only when dgl is present.

The loader samples minibatches with DGL on the CPU (CollateWrapper,
GIDS.py:143-201) and its iterator hands each batch to ``GIDS.fetch_feature``,
which appends the gathered feature tensor (``_PrefetchingIter``,
GIDS.py:204-258).
"""
from __future__ import annotations

import torch

from .GIDS import _PrefetchingIter


def make_dgl_loader(graph, indices, graph_sampler, batch_size, dim, gids, device=None, use_ddp=False, ddp_seed=0,
                    drop_last=False, shuffle=False, use_alternate_streams=None, **kwargs):
    try:
        import dgl  # noqa: F401
        from dgl.dataloading import create_tensorized_dataset, WorkerInitWrapper, remove_parent_storage_columns
        from dgl.utils import recursive_apply
    except ImportError as e:  # pragma: no cover - dgl is optional
        raise ImportError("GIDS_DGLDataLoader needs dgl; GIDS.fetch_feature works with any batch iterator") from e

    class CollateWrapper:
        def __init__(self, sample_func, g, dev):
            self.sample_func = sample_func
            self.g = g
            self.device = dev

        def __call__(self, items):
            items = recursive_apply(items, lambda x: x.to(self.device))
            batch = self.sample_func(self.g, items)
            return recursive_apply(batch, remove_parent_storage_columns, self.g)

    class Loader(torch.utils.data.DataLoader):
        def __init__(self):
            self.GIDS_Loader = gids
            self.dim = dim
            self.graph = graph
            self.indices = indices
            self.graph_sampler = graph_sampler
            idx = indices
            if isinstance(idx, dict):
                idx = {k: (v if torch.is_tensor(v) else torch.tensor(v)) for k, v in idx.items()}
            elif not torch.is_tensor(idx):
                idx = torch.tensor(idx)
            self.device = torch.device(device) if device is not None else torch.device("cpu")
            self.dataset = create_tensorized_dataset(idx, batch_size, drop_last, use_ddp, ddp_seed, shuffle,
                                                     kwargs.get("persistent_workers", False))
            self.shuffle = shuffle
            super().__init__(self.dataset, collate_fn=CollateWrapper(graph_sampler.sample, graph, self.device),
                             batch_size=None, pin_memory=False,
                             worker_init_fn=WorkerInitWrapper(kwargs.pop("worker_init_fn", None)), **kwargs)

        def __iter__(self):
            if self.shuffle:
                self.dataset.shuffle()
            return _PrefetchingIter(self, super().__iter__(), GIDS_Loader=self.GIDS_Loader)

        def print_stats(self):
            self.GIDS_Loader.print_stats()

        def print_timer(self):
            pass

    return Loader()
