// colmap.cu — COLMAP sparse models to the trainer's cameras and seed points (host code; replaces
// load_colmap_bundle, Sources/SplatXCore/ColmapLoader.cpp, and training_input_from_colmap,
// TrainingInput.cpp:10-47).
//
// Formats as COLMAP documents them: binary cameras.bin / images.bin / points3D.bin (little
// endian, u64 counts) or the text cameras.txt / images.txt (two lines per image) / points3D.txt
// ('#' comments, blank lines ignored, CRLF accepted); binary is used when cameras.bin exists.
// The trainer renders pure pinholes, so SIMPLE_PINHOLE (f, cx, cy) and PINHOLE (fx, fy, cx, cy)
// are accepted and every distortion model is rejected by name (the images must be undistorted
// first). Cameras: viewmat = [R(q) | t] with R from the normalised w-first world-to-camera
// quaternion in float, K from the intrinsics, image path = images_dir + "/" + name.
#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <memory>
#include <sstream>
#include <string>
#include <unordered_map>
#include <vector>

#include "sx_common.cuh"
#include "sx_internal.h"

namespace sx {

namespace {

// (name, parameter count) of COLMAP's camera models by model id
struct Model {
    const char* name;
    int params;
};
constexpr Model kModels[] = {{"SIMPLE_PINHOLE", 3}, {"PINHOLE", 4},         {"SIMPLE_RADIAL", 4},
                             {"RADIAL", 5},         {"OPENCV", 8},          {"OPENCV_FISHEYE", 8},
                             {"FULL_OPENCV", 12},   {"FOV", 5},             {"SIMPLE_RADIAL_FISHEYE", 4},
                             {"RADIAL_FISHEYE", 5}, {"THIN_PRISM_FISHEYE", 12}};
constexpr int kNumModels = sizeof(kModels) / sizeof(kModels[0]);

int model_params(int id) {
    if (id < 0 || id >= kNumModels) throw RuntimeError("colmap: unknown camera model " + std::to_string(id));
    return kModels[id].params;
}

void pinhole(SxColmap::Camera& c) {
    if (c.model == 0) {
        c.fx = c.fy = static_cast<float>(c.params[0]);
        c.cx = static_cast<float>(c.params[1]);
        c.cy = static_cast<float>(c.params[2]);
    } else if (c.model == 1) {
        c.fx = static_cast<float>(c.params[0]);
        c.fy = static_cast<float>(c.params[1]);
        c.cx = static_cast<float>(c.params[2]);
        c.cy = static_cast<float>(c.params[3]);
    } else {
        throw RuntimeError(std::string("colmap: unsupported camera model ") + kModels[c.model].name +
                           " — only PINHOLE / SIMPLE_PINHOLE are rendered; undistort the images "
                           "(e.g. COLMAP image_undistorter) into a PINHOLE model first");
    }
}

struct BinFile {
    FILE* f = nullptr;
    std::string path;
    explicit BinFile(const std::string& p) : f(std::fopen(p.c_str(), "rb")), path(p) {
        if (!f) throw RuntimeError("colmap: cannot open " + p);
    }
    ~BinFile() {
        if (f) std::fclose(f);
    }
    template <typename T>
    T get() {
        T v;
        if (std::fread(&v, sizeof(T), 1, f) != 1) throw RuntimeError("colmap: truncated " + path);
        return v;
    }
    void skip(uint64_t bytes) {
        if (std::fseek(f, static_cast<long>(bytes), SEEK_CUR) != 0)
            throw RuntimeError("colmap: seek failed " + path);
    }
    std::string cstr() {
        std::string s;
        for (;;) {
            const int ch = std::fgetc(f);
            if (ch == EOF) throw RuntimeError("colmap: truncated string " + path);
            if (ch == 0) return s;
            s.push_back(static_cast<char>(ch));
        }
    }
};

void load_bin(const std::string& dir, SxColmap& b) {
    {
        BinFile r(dir + "/cameras.bin");
        const uint64_t n = r.get<uint64_t>();
        for (uint64_t i = 0; i < n; ++i) {
            SxColmap::Camera c;
            c.id = r.get<int32_t>();
            c.model = r.get<int32_t>();
            c.width = static_cast<int64_t>(r.get<uint64_t>());
            c.height = static_cast<int64_t>(r.get<uint64_t>());
            c.params.resize(static_cast<size_t>(model_params(c.model)));
            for (double& p : c.params) p = r.get<double>();
            pinhole(c);
            b.cameras.push_back(std::move(c));
        }
    }
    {
        BinFile r(dir + "/images.bin");
        const uint64_t n = r.get<uint64_t>();
        for (uint64_t i = 0; i < n; ++i) {
            SxColmap::Image im;
            im.id = r.get<int32_t>();
            for (double& q : im.q) q = r.get<double>();
            for (double& t : im.t) t = r.get<double>();
            im.camera_id = r.get<int32_t>();
            im.name = r.cstr();
            r.skip(r.get<uint64_t>() * 24);  // POINTS2D: x f64, y f64, point3D id i64
            b.images.push_back(std::move(im));
        }
    }
    {
        BinFile r(dir + "/points3D.bin");
        const uint64_t n = r.get<uint64_t>();
        for (uint64_t i = 0; i < n; ++i) {
            (void)r.get<uint64_t>();  // point id
            for (int k = 0; k < 3; ++k) b.xyz.push_back(r.get<double>());
            for (int k = 0; k < 3; ++k) b.rgb.push_back(r.get<uint8_t>());
            (void)r.get<double>();        // reprojection error
            r.skip(r.get<uint64_t>() * 8);  // TRACK: image id i32, point2D index i32
        }
    }
}

struct TextFile {
    std::ifstream f;
    std::string path;
    long line = 0;
    explicit TextFile(const std::string& p) : f(p), path(p) {
        if (!f.is_open()) throw RuntimeError("colmap: cannot open " + p);
    }
    [[noreturn]] void fail(const std::string& m) const {
        throw RuntimeError("colmap: " + path + ":" + std::to_string(line) + ": " + m);
    }
    bool raw(std::string& s) {
        if (!std::getline(f, s)) return false;
        ++line;
        if (!s.empty() && s.back() == '\r') s.pop_back();
        return true;
    }
    bool data(std::string& s) {
        while (raw(s)) {
            const size_t i = s.find_first_not_of(" \t");
            if (i == std::string::npos || s[i] == '#') continue;
            return true;
        }
        return false;
    }
    long to_long(const std::string& tok, const char* what) const {
        errno = 0;
        char* end = nullptr;
        const long v = std::strtol(tok.c_str(), &end, 10);
        if (end == tok.c_str() || *end != '\0' || errno == ERANGE)
            fail(std::string("invalid ") + what + " '" + tok + "'");
        return v;
    }
    double to_double(const std::string& tok, const char* what) const {
        char* end = nullptr;
        const double v = std::strtod(tok.c_str(), &end);
        if (end == tok.c_str() || *end != '\0') fail(std::string("invalid ") + what + " '" + tok + "'");
        return v;
    }
};

std::vector<std::string> tokens(const std::string& s) {
    std::vector<std::string> out;
    std::istringstream is(s);
    std::string t;
    while (is >> t) out.push_back(t);
    return out;
}

void load_txt(const std::string& dir, SxColmap& b) {
    std::string ln;
    {
        TextFile r(dir + "/cameras.txt");
        while (r.data(ln)) {
            const auto t = tokens(ln);
            if (t.size() < 4)
                r.fail("expected CAMERA_ID MODEL WIDTH HEIGHT PARAMS[], got " +
                       std::to_string(t.size()) + " token(s)");
            SxColmap::Camera c;
            c.id = static_cast<int32_t>(r.to_long(t[0], "CAMERA_ID"));
            c.model = -1;
            for (int m = 0; m < kNumModels; ++m)
                if (t[1] == kModels[m].name) c.model = m;
            if (c.model < 0) r.fail("unknown camera model " + t[1]);
            c.width = r.to_long(t[2], "WIDTH");
            c.height = r.to_long(t[3], "HEIGHT");
            const int np = kModels[c.model].params;
            if (static_cast<int>(t.size()) - 4 != np)
                r.fail(t[1] + " expects " + std::to_string(np) + " params, got " +
                       std::to_string(t.size() - 4));
            for (int k = 0; k < np; ++k) c.params.push_back(r.to_double(t[4 + k], "PARAM"));
            pinhole(c);
            b.cameras.push_back(std::move(c));
        }
    }
    {
        TextFile r(dir + "/images.txt");
        while (r.data(ln)) {
            const auto t = tokens(ln);
            if (t.size() != 10)
                r.fail("expected 10 tokens (IMAGE_ID QW QX QY QZ TX TY TZ CAMERA_ID NAME), got " +
                       std::to_string(t.size()));
            SxColmap::Image im;
            im.id = static_cast<int32_t>(r.to_long(t[0], "IMAGE_ID"));
            for (int k = 0; k < 4; ++k) im.q[k] = r.to_double(t[1 + k], "QVEC");
            for (int k = 0; k < 3; ++k) im.t[k] = r.to_double(t[5 + k], "TVEC");
            im.camera_id = static_cast<int32_t>(r.to_long(t[8], "CAMERA_ID"));
            im.name = t[9];
            std::string points2d;  // the second line of every image (possibly empty)
            if (!r.raw(points2d)) r.fail("truncated: missing POINTS2D line after pose line");
            b.images.push_back(std::move(im));
        }
    }
    {
        TextFile r(dir + "/points3D.txt");
        while (r.data(ln)) {
            const auto t = tokens(ln);
            if (t.size() < 8)
                r.fail("expected POINT3D_ID X Y Z R G B ERROR TRACK[], got " +
                       std::to_string(t.size()) + " token(s)");
            if ((t.size() - 8) % 2 != 0)
                r.fail("TRACK[] must be (IMAGE_ID, POINT2D_IDX) pairs, got " +
                       std::to_string(t.size() - 8) + " trailing token(s)");
            (void)r.to_long(t[0], "POINT3D_ID");
            for (int k = 0; k < 3; ++k) b.xyz.push_back(r.to_double(t[1 + k], "XYZ"));
            for (int k = 0; k < 3; ++k) {
                const long v = r.to_long(t[4 + k], "RGB");
                if (v < 0 || v > 255) r.fail("RGB out of range 0..255: '" + t[4 + k] + "'");
                b.rgb.push_back(static_cast<uint8_t>(v));
            }
            (void)r.to_double(t[7], "ERROR");
        }
    }
}

bool exists(const std::string& p) {
    FILE* f = std::fopen(p.c_str(), "rb");
    if (!f) return false;
    std::fclose(f);
    return true;
}

}  // namespace

SxColmap* colmap_open(const char* sparse_dir, const char* images_dir) {
    if (!sparse_dir) throw_invalid("colmap_open", "null sparse_dir");
    std::unique_ptr<SxColmap> b(new SxColmap());
    const std::string dir(sparse_dir);
    if (exists(dir + "/cameras.bin")) load_bin(dir, *b);
    else if (exists(dir + "/cameras.txt")) load_txt(dir, *b);
    else throw RuntimeError("colmap: cannot open " + dir + "/cameras.{bin,txt}");
    b->images_dir = images_dir ? images_dir : "";
    std::unordered_map<int32_t, size_t> by_id;
    for (size_t i = 0; i < b->cameras.size(); ++i) by_id[b->cameras[i].id] = i;
    for (const auto& im : b->images)
        if (!by_id.count(im.camera_id))
            throw RuntimeError("training_input: image references unknown camera " +
                               std::to_string(im.camera_id));
    return b.release();
}

void colmap_cameras(const SxColmap& b, float* viewmats, float* Ks, int32_t* widths, int32_t* heights) {
    std::unordered_map<int32_t, const SxColmap::Camera*> by_id;
    for (const auto& c : b.cameras) by_id[c.id] = &c;
    for (size_t i = 0; i < b.images.size(); ++i) {
        const SxColmap::Image& im = b.images[i];
        const SxColmap::Camera& c = *by_id.at(im.camera_id);
        // the normalised quaternion's rotation in float (quat_to_rotmat, Math.cpp:9-18)
        float w = static_cast<float>(im.q[0]), x = static_cast<float>(im.q[1]);
        float y = static_cast<float>(im.q[2]), z = static_cast<float>(im.q[3]);
        const float n = std::sqrt(w * w + x * x + y * y + z * z);
        if (n > 0.0f) {
            w /= n;
            x /= n;
            y /= n;
            z /= n;
        }
        const float R[9] = {1 - 2 * (y * y + z * z), 2 * (x * y - w * z),     2 * (x * z + w * y),
                            2 * (x * y + w * z),     1 - 2 * (x * x + z * z), 2 * (y * z - w * x),
                            2 * (x * z - w * y),     2 * (y * z + w * x),     1 - 2 * (x * x + y * y)};
        float* vm = viewmats + i * 16;
        for (int r = 0; r < 3; ++r) {
            for (int k = 0; k < 3; ++k) vm[r * 4 + k] = R[r * 3 + k];
            vm[r * 4 + 3] = static_cast<float>(im.t[r]);
        }
        vm[12] = vm[13] = vm[14] = 0.0f;
        vm[15] = 1.0f;
        float* K = Ks + i * 9;
        const float k9[9] = {c.fx, 0.0f, c.cx, 0.0f, c.fy, c.cy, 0.0f, 0.0f, 1.0f};
        for (int k = 0; k < 9; ++k) K[k] = k9[k];
        widths[i] = static_cast<int32_t>(c.width);
        heights[i] = static_cast<int32_t>(c.height);
    }
}

}  // namespace sx
