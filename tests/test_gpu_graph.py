"""Frame graphs (KT_GS_FLAG_GRAPH): a path's frame captured once as a CUDA graph and replayed with
new cameras must draw exactly what the stream-launched frame draws, and must be captured again
when anything it bakes in changes (image pointer, scene, buffers after a capacity growth)."""

import numpy as np
import pytest

from klartraum_b200 import Renderer, make_scene, native as N, orbit_views

from helpers import background

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

W, H = 640, 360


def _scene(n=60000, seed=21):
    return make_scene("single_1m", n=n, seed=seed)


@pytest.mark.parametrize("extra", [0, N.FLAG_SORTED_KEYS], ids=["placed", "sorted_keys"])
def test_graph_replays_match_stream_frames(extra):
    g3d = _scene()
    cams = orbit_views(5, 2.5, W, H, fovy_deg=60.0)
    bg = torch.from_numpy(background(H, W, "random")).cuda()
    ref, got = [], []
    for flags, out in ((extra, ref), (extra | N.FLAG_GRAPH, got)):
        r = Renderer(W, H, bin_size=16, sh_degree=3, flags=flags)
        r.set_gaussians(g3d)
        img = bg.clone()
        for c in cams:  # the same image buffer every frame: one capture, replays after it
            img.copy_(bg)
            r.render(c, img)
            out.append(img.clone())
        r.close()
    for a, b in zip(ref, got):
        assert torch.equal(a, b)


def test_graph_replays_in_flight_keep_their_cameras():
    """Replays of one path's graph enqueued back to back, each with its own camera (set as the
    projection kernel's argument in the executable graph) and no wait between them: every frame
    draws its own view."""
    g3d = _scene(n=30000)
    cams = orbit_views(5, 2.5, W, H, fovy_deg=60.0)
    bgh = background(H, W, "random")
    r = Renderer(W, H, bin_size=16, sh_degree=3)
    r.set_gaussians(g3d)
    ref = [r.render_host(c, bgh.copy()) for c in cams]
    r.set_flags(N.FLAG_GRAPH | N.FLAG_ASYNC)
    stream = torch.cuda.Stream()
    hosts = [torch.from_numpy(bgh.copy()).pin_memory() for _ in cams]
    for c, h in zip(cams, hosts):
        r.render_host(c, h.data_ptr(), stream=stream.cuda_stream)
    r.sync()
    for a, h in zip(ref, hosts):
        assert np.array_equal(a, h.numpy())
    assert len({h.numpy().tobytes() for h in hosts}) == len(cams)
    r.close()


def test_graph_recaptures_on_new_image_scene_and_capacity():
    g3d, g3d_b = _scene(seed=21), _scene(n=40000, seed=22)
    cams = orbit_views(3, 2.5, W, H, fovy_deg=60.0)
    bg = torch.from_numpy(background(H, W)).cuda()

    def plain(scene, cam):
        r = Renderer(W, H, bin_size=16, sh_degree=3)
        r.set_gaussians(scene)
        img = bg.clone()
        r.render(cam, img)
        r.close()
        return img

    # a capacity far too small: the first replay overflows, the buffers grow, the graph is
    # captured again and the frame is drawn
    r = Renderer(W, H, bin_size=16, sh_degree=3, flags=N.FLAG_GRAPH, key_capacity=4096)
    r.set_gaussians(g3d)
    a = bg.clone()
    r.render(cams[0], a)
    assert r.stats()["key_capacity"] >= r.stats()["num_keys"] > 4096
    assert torch.equal(a, plain(g3d, cams[0]))
    # another output buffer
    b = bg.clone()
    r.render(cams[1], b)
    assert torch.equal(b, plain(g3d, cams[1]))
    # another scene
    r.set_gaussians(g3d_b)
    c = bg.clone()
    r.render(cams[2], c)
    assert torch.equal(c, plain(g3d_b, cams[2]))
    # back to the first buffer, async replays, one sync at the end
    r.set_flags(N.FLAG_GRAPH | N.FLAG_ASYNC)
    for _ in range(20):
        a.copy_(bg)
        r.render(cams[1], a)
    r.sync()
    assert torch.equal(a, plain(g3d_b, cams[1]))
    assert r.counters()["frames"] >= 20
    r.close()


def test_graph_render_host():
    g3d = _scene(n=20000)
    cam = orbit_views(1, 2.5, W, H, fovy_deg=60.0)[0]
    bgh = background(H, W, "random")
    outs = []
    for flags in (0, N.FLAG_GRAPH):
        r = Renderer(W, H, bin_size=16, sh_degree=3, flags=flags)
        r.set_gaussians(g3d)
        host = bgh.copy()
        r.render_host(cam, host)
        host2 = bgh.copy()
        r.render_host(cam, host2)  # the second call replays
        outs.append((host, host2))
        r.close()
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])


@pytest.mark.parametrize("flags", [0, N.FLAG_GRAPH], ids=["stream", "graph"])
def test_async_render_host_frames_in_flight(flags):
    """kt_gs_render_host with KT_GS_FLAG_ASYNC: three paths on three streams, each host image read
    only after kt_gs_sync(path); every image equals the synchronous render of its view."""
    g3d = _scene(n=30000)
    cams = orbit_views(7, 2.5, W, H, fovy_deg=60.0)
    bgh = background(H, W, "random")
    ref = []
    r = Renderer(W, H, bin_size=16, sh_degree=3)
    r.set_gaussians(g3d)
    for c in cams:
        ref.append(r.render_host(c, bgh.copy()))
    r.close()
    r = Renderer(W, H, bin_size=16, sh_degree=3, num_paths=3)
    r.set_gaussians(g3d)
    img = torch.from_numpy(bgh).cuda()
    for p in range(3):  # checked frames size every path's buffers (async frames cannot grow)
        for c in cams:
            r.render(c, img, path=p)
    r.set_flags(flags | N.FLAG_ASYNC)
    streams = [torch.cuda.Stream() for _ in range(3)]
    hosts = [torch.empty((H, W, 4), dtype=torch.uint8, pin_memory=True) for _ in range(3)]
    got = [None] * len(cams)
    for i, c in enumerate(cams):
        p = i % 3
        if i >= 3:
            r.sync(p)
            got[i - 3] = hosts[p].numpy().copy()
        hosts[p].copy_(torch.from_numpy(bgh))
        r.render_host(c, hosts[p].data_ptr(), path=p, stream=streams[p].cuda_stream)
    for i in range(len(cams) - 3, len(cams)):
        r.sync(i % 3)
        got[i] = hosts[i % 3].numpy().copy()
    r.close()
    for a, b in zip(ref, got):
        assert np.array_equal(a, b)
