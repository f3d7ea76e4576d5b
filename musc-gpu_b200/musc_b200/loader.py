"""Pool-image loading for the ``b200`` backend: host decode, device preprocessing.

The reference decodes, resizes and normalises every image on the host
(``datasets/mvtec.py:98-99`` with the CLIP evaluation transform,
``models/backbone/open_clip/transform.py:124-133``), collates fp32 batches in
worker threads (``models/modules/_loader.py:8-43``), pins them and copies them
to the device (``models/musc.py:197``).  Here the host threads only decode
(``RawRGB`` replaces the dataset's ``clip_transformer``); each batch's 8-bit
pixels go through one pinned staging buffer to the device on a copy stream, and
``musc_b200_preprocess_images`` resizes and normalises them there, bit for bit
with the reference's fp32 tensors.  The copy moves 3 bytes per input pixel
(2.4 MB for a 900 x 900 MVTec image) instead of 12 per output pixel (3.2 MB),
and the host's resize, which costs tens of milliseconds per image, is gone.

``DeviceImageLoader`` keeps ``ThreadedDatasetLoader``'s contract: batches in
dataset order, ``batch_size * prefetch_batches`` items in flight, worker
exceptions raised to the caller, ``len()`` in batches, and the collated item
dict -- with ``"image"`` a ``(B, 3, S, S)`` device tensor on the current stream.
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor
from typing import Iterator, Sequence

import numpy as np
import torch
from torch.utils.data._utils.collate import default_collate
from torch.utils.data._utils.pin_memory import pin_memory as pin_batch

from . import ops


class RawRGB:
    """Drop-in for the dataset's ``clip_transformer``: the decoded image as an
    ``(H, W, 3)`` uint8 array (``_convert_to_rgb`` of ``transform.py:52-53``), with the
    resize and normalisation left to the device."""

    def __call__(self, image) -> np.ndarray:
        if image.mode != 'RGB':
            image = image.convert('RGB')
        return np.asarray(image, dtype=np.uint8)


def ordered_batches(dataset, batch_size: int, workers: int, prefetch_batches: int) -> Iterator[list]:
    """Items of ``dataset`` in order, ``batch_size`` at a time, loaded by ``workers`` threads
    with at most ``batch_size * prefetch_batches`` items in flight; a worker's exception is
    raised here (``_loader.py:21-43``)."""
    with ThreadPoolExecutor(max_workers=workers) as executor:
        indices = iter(range(len(dataset)))
        pending = []
        for _ in range(batch_size * prefetch_batches):
            index = next(indices, None)
            if index is None:
                break
            pending.append(executor.submit(dataset.__getitem__, index))
        while pending:
            take = min(batch_size, len(pending))
            samples = [future.result() for future in pending[:take]]
            del pending[:take]
            for _ in range(take):
                index = next(indices, None)
                if index is None:
                    break
                pending.append(executor.submit(dataset.__getitem__, index))
            yield samples


def _image_of(sample):
    return sample['image'] if isinstance(sample, dict) else sample


def _as_hwc_u8(image) -> np.ndarray:
    arr = image.numpy() if isinstance(image, torch.Tensor) else np.asarray(image)
    if arr.dtype != np.uint8 or arr.ndim != 3 or arr.shape[2] != 3:
        raise ValueError('DeviceImageLoader: items must carry (H, W, 3) uint8 images (use RawRGB as the '
                         'dataset transform)')
    return arr


class DeviceImageLoader:
    """``ThreadedDatasetLoader`` (``models/modules/_loader.py:8-43``) whose batches are
    preprocessed on the device.  ``size``, ``filter``, ``mean`` and ``std`` are the
    transform's (CLIP evaluation defaults: 518, bicubic, OpenAI constants)."""

    def __init__(self, dataset, batch_size: int = 4, workers: int = 4, prefetch_batches: int = 2,
                 pin_memory: bool = True, device=None, size: int = 518, filter: str = 'bicubic',
                 mean: Sequence[float] = ops.OPENAI_MEAN, std: Sequence[float] = ops.OPENAI_STD,
                 out_dtype: torch.dtype = torch.float32):
        if batch_size < 1 or workers < 1 or prefetch_batches < 1:
            raise ValueError('Loader sizes must be positive')
        if filter not in ('bicubic', 'bilinear'):
            raise ValueError("filter must be 'bicubic' or 'bilinear'")
        self.dataset = dataset
        self.batch_size = batch_size
        self.workers = workers
        self.prefetch_batches = prefetch_batches
        self.pin_memory = pin_memory
        self.device = torch.device(device) if device is not None else torch.device('cuda', torch.cuda.current_device())
        self.size = size
        self.filter = filter
        self.mean, self.std = tuple(mean), tuple(std)
        self.out_dtype = out_dtype
        self._staging: list[torch.Tensor | None] = [None, None]
        self._copied: list[torch.cuda.Event | None] = [None, None]
        self._copy_stream: torch.cuda.Stream | None = None
        self._copier: ThreadPoolExecutor | None = None

    def __len__(self) -> int:
        return (len(self.dataset) + self.batch_size - 1) // self.batch_size

    def _stage(self, slot: int, nbytes: int) -> torch.Tensor:
        """Pinned staging buffer ``slot``, free to overwrite (its last copy has finished)."""
        if self._copied[slot] is not None:
            self._copied[slot].synchronize()
        buf = self._staging[slot]
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(nbytes, dtype=torch.uint8, pin_memory=self.pin_memory)
            self._staging[slot] = buf
        return buf

    _CHUNK = 16   # images per host copy / H2D / kernel step of the pipeline below

    def _runs(self, arrays):
        """(start, end, h, w): runs of equal-sized images, at most ``_CHUNK`` long."""
        start = 0
        while start < len(arrays):
            h, w, _ = arrays[start].shape
            end = start + 1
            while end < len(arrays) and end - start < self._CHUNK and arrays[end].shape == (h, w, 3):
                end += 1
            yield start, end, h, w
            start = end

    def preprocess(self, images: list, slot: int = 0) -> torch.Tensor:
        """``images`` (decoded ``(H, W, 3)`` uint8 arrays) -> ``(B, 3, S, S)`` on the device,
        ordered on the current stream.

        Pipelined in runs of up to 16 equal-sized images: the host threads copy a run into
        the pinned staging buffer while the copy stream moves the previous run to the device
        and the current stream resamples the one before."""
        arrays = [_as_hwc_u8(im) for im in images]
        dev = self.device
        if self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(device=dev)
            self._copier = ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1))
        nbytes = sum(a.nbytes for a in arrays)
        host = self._stage(slot, nbytes)
        compute = torch.cuda.current_stream(dev)
        with torch.cuda.device(dev):
            out = torch.empty((len(arrays), 3, self.size, self.size), dtype=self.out_dtype, device=dev)
            with torch.cuda.stream(self._copy_stream):
                # allocated on the copy stream, so the copies wait for nothing on the compute
                # stream; record_stream keeps it alive until the compute stream is done with it
                staged = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            staged.record_stream(compute)
            offset = 0
            for start, end, h, w in self._runs(arrays):
                size = (end - start) * h * w * 3
                dst = host[offset:offset + size].numpy().reshape(end - start, h, w, 3)
                list(self._copier.map(lambda j: np.copyto(dst[j], arrays[start + j]), range(end - start)))
                with torch.cuda.stream(self._copy_stream):
                    staged[offset:offset + size].copy_(host[offset:offset + size], non_blocking=True)
                    done = torch.cuda.Event()
                    done.record(self._copy_stream)
                self._copied[slot] = done   # copies are ordered: the last event covers them all
                compute.wait_event(done)
                run = staged[offset:offset + size].view(end - start, h, w, 3)
                ops.preprocess_images(run, self.size, self.filter, self.mean, self.std, self.out_dtype,
                                      out=out[start:end])
                offset += size
        return out

    def close(self) -> None:
        """Wait for the staging copies in flight and stop the host copy threads."""
        for ev in self._copied:
            if ev is not None:
                ev.synchronize()
        if self._copier is not None:
            self._copier.shutdown(wait=True)
            self._copier = None
            self._copy_stream = None

    def __iter__(self):
        for i, samples in enumerate(ordered_batches(self.dataset, self.batch_size, self.workers,
                                                    self.prefetch_batches)):
            images = self.preprocess([_image_of(s) for s in samples], slot=i % 2)
            if isinstance(samples[0], dict):
                rest = default_collate([{k: v for k, v in s.items() if k != 'image'} for s in samples])
                if self.pin_memory:
                    rest = pin_batch(rest)
                rest['image'] = images
                yield rest
            else:
                yield images
