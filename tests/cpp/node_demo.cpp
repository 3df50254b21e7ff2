// Renders one frame through the C++ node interface (include/kt_gs_node.hpp) the way klartraum
// code drives VulkanGaussianSplatting: build the node from an image source and a camera UBO,
// compile a ComputeGraph from it, submit a path. Also checks the reference's checkInput errors
// (src/vulkan_gaussian_splatting.cpp:220-232).
//   node_demo <scene.bin> <camera.bin> <width> <height> <out.rgba>
#include <cstdio>
#include <fstream>
#include <iterator>
#include <vector>

#include "kt_gs_node.hpp"

template <class T>
static std::vector<T> read_all(const char* path) {
    std::ifstream f(path, std::ios::binary);
    std::vector<char> raw((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    std::vector<T> out(raw.size() / sizeof(T));
    if (!out.empty()) std::memcpy(out.data(), raw.data(), out.size() * sizeof(T));
    return out;
}

int main(int argc, char** argv) {
    if (argc != 6) {
        std::fprintf(stderr, "usage: node_demo scene.bin camera.bin width height out.rgba\n");
        return 64;
    }
    auto gaussians = read_all<kt_gaussian3d>(argv[1]);
    auto cams = read_all<kt_camera_mvp>(argv[2]);
    const uint32_t W = (uint32_t)std::atoi(argv[3]), H = (uint32_t)std::atoi(argv[4]);
    if (cams.empty()) return 65;

    klartraum::CudaContext context(0);
    auto image = std::make_shared<klartraum::ImageViewSrc>(W, H, 2);
    auto camera = std::make_shared<klartraum::CameraUboType>();
    kt_gs_config cfg;
    kt_gs_config_default(&cfg);
    cfg.bin_width = cfg.bin_height = 16;
    cfg.sh_degree = -1;
    cfg.num_paths = 2;
    auto node = std::make_shared<klartraum::VulkanGaussianSplatting>(context, image, camera, gaussians, &cfg);

    int bad = 0;
    try { node->setInput(camera, 0); bad |= 1; } catch (const std::runtime_error&) {}
    try { node->setInput(image, 1); bad |= 2; } catch (const std::runtime_error&) {}
    try { node->setInput(image, 2); bad |= 4; } catch (const std::runtime_error&) {}
    if (bad) return 10 + bad;
    if (std::string(node->getType()) != "GaussianSplatting") return 20;

    klartraum::ComputeGraph graph(context, 2);
    graph.compileFrom(node);
    if (graph.order().size() != 3 || graph.order().back() != node) return 21;

    camera->ubo = cams[0];
    camera->update(0);
    camera->update(1);
    cudaStream_t stream;
    cudaStreamCreate(&stream);
    graph.submitAndWait(stream, 0);
    graph.submitAndWait(stream, 1);
    auto a = image->download(0), b = image->download(1);
    if (a != b) return 22;
    std::ofstream out(argv[5], std::ios::binary);
    out.write(reinterpret_cast<const char*>(a.data()), (std::streamsize)a.size());
    cudaStreamDestroy(stream);
    std::printf("%s rendered %ux%u from %zu Gaussians\n", node->getType(), W, H, gaussians.size());
    return 0;
}
