"""Image crops of the training and evaluation transforms (the ADM recipe of openai/guided-diffusion
image_datasets.py, as the reference uses it in baselines/PixelGen/src/data/dataset/augmentation.py:8-79):
box-halve while the short side is at least twice the target, bicubic-resize the short side to the target (eval) or to
a random size in [size/max_frac, size/min_frac] (train), then crop (center / random)."""
import math
import random

import numpy as np
from PIL import Image


def _halve(img, target):
    while min(*img.size) >= 2 * target:
        img = img.resize(tuple(x // 2 for x in img.size), resample=Image.BOX)
    return img


def center_crop_arr(pil_image, image_size):
    img = _halve(pil_image, image_size)
    scale = image_size / min(*img.size)
    img = img.resize(tuple(round(x * scale) for x in img.size), resample=Image.BICUBIC)
    arr = np.array(img)
    y, x = (arr.shape[0] - image_size) // 2, (arr.shape[1] - image_size) // 2
    return Image.fromarray(arr[y:y + image_size, x:x + image_size])


def random_crop_arr(pil_image, image_size, min_crop_frac=0.8, max_crop_frac=1.0, rng=random):
    smaller = rng.randrange(math.ceil(image_size / max_crop_frac), math.ceil(image_size / min_crop_frac) + 1)
    img = _halve(pil_image, smaller)
    scale = smaller / min(*img.size)
    img = img.resize(tuple(round(x * scale) for x in img.size), resample=Image.BICUBIC)
    arr = np.array(img)
    y = rng.randrange(arr.shape[0] - image_size + 1)
    x = rng.randrange(arr.shape[1] - image_size + 1)
    return Image.fromarray(arr[y:y + image_size, x:x + image_size])


def decode_center_u8(image_bytes, image_size=256):
    """Encoded image -> center-cropped uint8 HWC array (the evaluation transform before ToTensor)."""
    import io
    return np.asarray(center_crop_arr(Image.open(io.BytesIO(image_bytes)).convert("RGB"), image_size), dtype=np.uint8)
