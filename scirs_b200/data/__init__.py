"""Datasets, the native-prefetching DataLoader and batch transforms."""
from .loader import (DataLoader, Dataset, GaussianNoise, InMemoryDataset, Normalize, RandomCrop,
                     RandomHorizontalFlip)
