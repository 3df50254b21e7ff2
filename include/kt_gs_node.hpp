// kt_gs_node.hpp - header-only C++ graph-node interface over the C ABI (kt_gs.h).
//
// Mirrors the part of klartraum's compute-graph API that the Gaussian-splatting node lives in,
// so that C++ code written against VulkanGaussianSplatting keeps its shape:
//   ComputeGraphElement     include/klartraum/computegraph/computegraphelement.hpp:30-102
//   ComputeGraphGroup       include/klartraum/computegraph/computegraphgroup.hpp:7-23
//   RenderGraphElement      include/klartraum/computegraph/rendergraphelement.hpp:9-21
//   UniformBufferObject<T>  include/klartraum/computegraph/uniformbufferobject.hpp:22-199
//   ImageViewSrc            include/klartraum/computegraph/imageviewsrc.hpp:13-55
//   GaussianSplatting       include/klartraum/vulkan_gaussian_splatting.hpp:23-83
//   ComputeGraph            include/klartraum/computegraph/computegraph.hpp:69-160, 344-411
// A Vulkan command buffer becomes a CUDA stream, a VulkanContext a CudaContext (device index),
// a swap-chain image a headless RGBA8 device image per path. Errors are std::runtime_error,
// as in the reference.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <memory>
#include <queue>
#include <stdexcept>
#include <string>
#include <vector>

#include "kt_gs.h"

namespace klartraum {

// CUDA device the graph runs on (the reference's VulkanContext).
class CudaContext {
public:
    explicit CudaContext(int device = 0) : device_(device) {
        if (cudaSetDevice(device) != cudaSuccess) throw std::runtime_error("cannot select CUDA device");
    }
    int getDevice() const { return device_; }

private:
    int device_;
};

inline void ktCheck(kt_status s, const kt_gs_ctx* ctx = nullptr) {
    if (s != KT_OK) {
        std::string msg = kt_gs_status_string(s);
        if (ctx) msg += std::string(": ") + kt_gs_last_error(ctx);
        throw std::runtime_error(msg);
    }
}

class ComputeGraphElement;
typedef std::shared_ptr<ComputeGraphElement> ComputeGraphElementPtr;

class ComputeGraphElement : public std::enable_shared_from_this<ComputeGraphElement> {
public:
    virtual ~ComputeGraphElement() = default;

    void setInput(ComputeGraphElementPtr input, int index = 0, int slot = -1) {
        if (slot == -1)
            checkInput(input, index);
        else
            checkInput(input->getInputElement(slot), index);
        inputs[index] = input;
        srcOutputSlots[index] = slot;
    }

    virtual void checkInput(ComputeGraphElementPtr, int = 0) {
        throw std::runtime_error("checkInput not implemented for this element");
    }

    ComputeGraphElementPtr getInputElement(int index = 0) {
        if (srcOutputSlots[index] != -1) return inputs[index]->getInputElement(srcOutputSlots[index]);
        return inputs[index];
    }

    virtual void _setup(CudaContext&, uint32_t) { initialized = true; }

    virtual void _record(cudaStream_t, uint32_t) {
        if (!initialized) throw std::runtime_error("ComputeGraphElement not initialized");
    }

    virtual const char* getType() const = 0;
    virtual const char* getName() const { return name.c_str(); }
    virtual std::map<int, ComputeGraphElementPtr> getInputs() const { return inputs; }
    void setName(const std::string& n) { name = n; }

protected:
    std::map<int, ComputeGraphElementPtr> inputs;
    std::map<int, int> srcOutputSlots;
    bool initialized = false;
    std::string name;
};

class ComputeGraphGroup : public virtual ComputeGraphElement {
public:
    const char* getType() const override { return "ComputeGraphGroup"; }
    std::map<int, ComputeGraphElementPtr> getInputs() const override { return outputElements; }

protected:
    std::map<int, ComputeGraphElementPtr> outputElements;
};

// CameraMVP (include/klartraum/camera.hpp:44-48), column-major float[16] per matrix.
typedef kt_camera_mvp CameraMVP;

template <class T>
class UniformBufferObject : public virtual ComputeGraphElement {
public:
    void _setup(CudaContext&, uint32_t numberPaths) override {
        perPath.assign(numberPaths, ubo);
        initialized = true;
    }
    const char* getType() const override { return "UniformBufferObject"; }
    // uniformbufferobject.hpp:67-70: copy the host-side ubo into the path's buffer
    void update(uint32_t pathId) {
        if (pathId >= perPath.size()) perPath.resize(pathId + 1, ubo);
        perPath[pathId] = ubo;
    }
    const T& get(uint32_t pathId) const { return perPath.at(pathId); }
    T ubo{};

private:
    std::vector<T> perPath;
};

typedef UniformBufferObject<CameraMVP> CameraUboType;

class RenderGraphElement : public virtual ComputeGraphElement {
public:
    std::shared_ptr<CameraUboType> getCameraUBO() {
        for (auto& input : inputs) {
            auto ubo = std::dynamic_pointer_cast<CameraUboType>(input.second);
            if (ubo) return ubo;
        }
        throw std::runtime_error("No CameraUboType found in inputs!");
    }
};

// Headless RGBA8 device images, one per path, cleared to (0,0,0,1) like the reference's
// render pass (include/klartraum/computegraph/renderpass.hpp:170).
class ImageViewSrc : public virtual ComputeGraphElement {
public:
    ImageViewSrc(uint32_t width, uint32_t height, uint32_t numberPaths = 1) : w(width), h(height) {
        for (uint32_t p = 0; p < numberPaths; ++p) {
            void* d = nullptr;
            if (cudaMalloc(&d, bytes()) != cudaSuccess) throw std::runtime_error("cannot allocate image");
            images.push_back(d);
        }
        clear();
    }
    ~ImageViewSrc() override {
        for (void* d : images) cudaFree(d);
    }
    const char* getType() const override { return "ImageViewSrc"; }
    void* getImage(uint32_t pathId) {
        if (pathId >= images.size()) throw std::runtime_error("pathId out of range!");
        return images[pathId];
    }
    void clear() {
        std::vector<unsigned char> px(bytes(), 0);
        for (size_t i = 3; i < px.size(); i += 4) px[i] = 255;
        for (void* d : images) cudaMemcpy(d, px.data(), px.size(), cudaMemcpyHostToDevice);
    }
    std::vector<unsigned char> download(uint32_t pathId) {
        std::vector<unsigned char> px(bytes());
        if (cudaMemcpy(px.data(), getImage(pathId), px.size(), cudaMemcpyDeviceToHost) != cudaSuccess)
            throw std::runtime_error("image download failed");
        return px;
    }
    uint32_t width() const { return w; }
    uint32_t height() const { return h; }

private:
    size_t bytes() const { return (size_t)w * h * 4; }
    uint32_t w, h;
    std::vector<void*> images;
};

// The node: input 0 = ImageViewSrc, input 1 = CameraUboType; renders the scene into the
// path's image on _record. Extra constructor arguments are the renderer configuration.
class GaussianSplatting : public virtual RenderGraphElement, public virtual ComputeGraphGroup {
public:
    GaussianSplatting(CudaContext& context, std::shared_ptr<ImageViewSrc> imageViewSrc,
                      std::shared_ptr<CameraUboType> cameraUBO, std::string path,
                      const kt_gs_config* cfg = nullptr)
        : GaussianSplatting(context, imageViewSrc, cameraUBO, cfg) {
        ktCheck(kt_gs_load_spz(ctx, path.c_str()), ctx);
    }

    GaussianSplatting(CudaContext& context, std::shared_ptr<ImageViewSrc> imageViewSrc,
                      std::shared_ptr<CameraUboType> cameraUBO, const std::vector<kt_gaussian3d>& gaussians,
                      const kt_gs_config* cfg = nullptr)
        : GaussianSplatting(context, imageViewSrc, cameraUBO, cfg) {
        ktCheck(kt_gs_set_gaussians(ctx, gaussians.data(), gaussians.size()), ctx);
    }

    ~GaussianSplatting() override {
        if (ctx) kt_gs_destroy(ctx);
    }

    // The reference's scene loaders (src/vulkan_gaussian_splatting.cpp:322-417), replacing the scene.
    void loadSPZModel(const std::string& path) { ktCheck(kt_gs_load_spz(ctx, path.c_str()), ctx); }
    void loadPLYModel(const std::string& path) { ktCheck(kt_gs_load_ply(ctx, path.c_str()), ctx); }

    // src/vulkan_gaussian_splatting.cpp:220-232
    void checkInput(ComputeGraphElementPtr input, int index = 0) override {
        if (index == 0 && !std::dynamic_pointer_cast<ImageViewSrc>(input))
            throw std::runtime_error("input is not an ImageViewSrc!");
        if (index == 1 && !std::dynamic_pointer_cast<CameraUboType>(input))
            throw std::runtime_error("input is not a CameraUboType!");
        if (index > 1) throw std::runtime_error("input index out of range!");
    }

    void _setup(CudaContext&, uint32_t numberPaths) override {
        numberOfPaths = numberPaths;
        initialized = true;
    }

    void _record(cudaStream_t stream, uint32_t pathId) override {
        auto image = std::dynamic_pointer_cast<ImageViewSrc>(getInputElement(0));
        if (!image) throw std::runtime_error("input is not an ImageViewSrc!");
        auto camera = std::dynamic_pointer_cast<CameraUboType>(getInputElement(1));
        const uint32_t slot = pathId % config.num_paths;
        ktCheck(kt_gs_render(ctx, &camera->get(pathId), image->getImage(pathId), slot, stream), ctx);
    }

    const char* getType() const override { return "GaussianSplatting"; }
    // The node draws itself, so the graph reaches its image and camera through it (the
    // reference's group exposes its internal splat element instead, .cpp:212).
    std::map<int, ComputeGraphElementPtr> getInputs() const override { return inputs; }
    kt_gs_ctx* handle() const { return ctx; }

private:
    GaussianSplatting(CudaContext& context, std::shared_ptr<ImageViewSrc> imageViewSrc,
                      std::shared_ptr<CameraUboType> cameraUBO, const kt_gs_config* cfg) {
        if (cfg) {
            config = *cfg;
        } else {
            kt_gs_config_default(&config);
        }
        config.width = imageViewSrc->width();
        config.height = imageViewSrc->height();
        setInput(imageViewSrc, 0);
        setInput(cameraUBO, 1);
        ktCheck(kt_gs_create(&config, context.getDevice(), &ctx));
    }

    kt_gs_config config{};
    kt_gs_ctx* ctx = nullptr;
    uint32_t numberOfPaths = 0;
};

// Name of the reference class, for code that spells it out.
typedef GaussianSplatting VulkanGaussianSplatting;

// Headless graph runner: orders the elements reachable from the output with Kahn's algorithm
// (computegraph.hpp:344-411), sets them up for numberPaths paths and, per submit, records
// every element of the path on a CUDA stream in that order.
class ComputeGraph {
public:
    ComputeGraph(CudaContext& context, uint32_t numberPaths = 1) : ctx(context), paths(numberPaths) {}

    void compileFrom(ComputeGraphElementPtr element) {
        computeOrder(element);
        for (auto& e : ordered) e->_setup(ctx, paths);
    }

    void submitTo(cudaStream_t stream, uint32_t pathId) {
        if (pathId >= paths) throw std::runtime_error("pathId out of range!");
        for (auto& e : ordered) e->_record(stream, pathId);
    }

    void submitAndWait(cudaStream_t stream, uint32_t pathId) {
        submitTo(stream, pathId);
        if (cudaStreamSynchronize(stream) != cudaSuccess) throw std::runtime_error("stream synchronisation failed");
    }

    const std::vector<ComputeGraphElementPtr>& order() const { return ordered; }

private:
    typedef std::map<ComputeGraphElementPtr, std::vector<ComputeGraphElementPtr>> EdgeList;

    void fillEdges(EdgeList& edges, EdgeList& incoming, ComputeGraphElementPtr element) {
        for (auto& input : element->getInputs()) {
            auto& out = edges[element];
            if (std::find(out.begin(), out.end(), input.second) == out.end()) {
                out.push_back(input.second);
                incoming[input.second].push_back(element);
                fillEdges(edges, incoming, input.second);
            }
        }
    }

    void computeOrder(ComputeGraphElementPtr element) {
        ordered.clear();
        EdgeList edges, incoming;
        fillEdges(edges, incoming, element);
        std::queue<ComputeGraphElementPtr> S;
        S.push(element);
        while (!S.empty()) {
            auto n = S.front();
            S.pop();
            ordered.push_back(n);
            for (auto& input : n->getInputs()) {
                auto m = input.second;
                auto& out = edges[n];
                auto it = std::find(out.begin(), out.end(), m);
                if (it == out.end()) continue;
                out.erase(it);
                auto& inc = incoming[m];
                inc.erase(std::find(inc.begin(), inc.end(), n));
                if (inc.empty()) S.push(m);
            }
        }
        for (auto& e : edges)
            if (!e.second.empty()) throw std::runtime_error("graph has cycles!");
        std::reverse(ordered.begin(), ordered.end());
    }

    CudaContext& ctx;
    uint32_t paths;
    std::vector<ComputeGraphElementPtr> ordered;
};

}  // namespace klartraum
