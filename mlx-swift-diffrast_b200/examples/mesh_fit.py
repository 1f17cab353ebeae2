"""Runs the reference's MeshFitExample on the GPU and prints the loss
curve; with --out PATH writes the final target|current frame as a PPM."""
import argparse

import fits

if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--out", default=None)
    a = ap.parse_args()
    losses, final, target, tgt_img, cur_img = fits.run_mesh(a.steps)
    for i, l in enumerate(losses, 1):
        if i == 1 or i % 20 == 0 or i == len(losses):
            print(f"  step {i:4d}  loss = {l:.6f}")
    d = (final - target)[0]
    print("final minus target (first two components per vertex):")
    for v in range(d.shape[0]):
        print(f"  v{v}  ({d[v, 0]:+.4f}, {d[v, 1]:+.4f})")
    if a.out:
        fits.write_side_by_side(a.out, tgt_img, cur_img)
        print("wrote", a.out)
