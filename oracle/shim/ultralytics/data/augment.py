"""Shim: ``classify_transforms`` as ultralytics defines it for inference at size S —
torchvision Resize(S, bilinear; PIL antialiased) of the shortest edge, CenterCrop(S),
ToTensor (/255), Normalize with mean 0 / std 1 (DEFAULT_MEAN / DEFAULT_STD)."""
import torchvision.transforms as T


def classify_transforms(size=224, **_):
    return T.Compose([T.Resize(size, interpolation=T.InterpolationMode.BILINEAR),
                      T.CenterCrop(size), T.ToTensor(),
                      T.Normalize(mean=(0.0, 0.0, 0.0), std=(1.0, 1.0, 1.0))])
