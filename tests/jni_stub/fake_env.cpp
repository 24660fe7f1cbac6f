// Fake JNIEnv for the CPU test of the JNI glue (see jni.h beside this file):
// arrays are host vectors, strings are C strings, ThrowNew records the
// exception class and message.  main() drives the glue's entry points that
// need no GPU and prints one line per check; the test compares them.
#include <jni.h>

#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

struct FakeArray : _jobject {
    std::vector<uint8_t> bytes;
    jsize len = 0;
};
struct FakeString : _jobject {
    std::string s;
};
struct FakeClass : _jobject {
    std::string name;
};

static std::string g_thrown_class, g_thrown_msg;
static FakeClass g_classes[8];
static int g_nclass = 0;

jclass JNIEnv::FindClass(const char* name) {
    FakeClass* c = &g_classes[g_nclass++ % 8];
    c->name = name;
    return c;
}
jint JNIEnv::ThrowNew(jclass cls, const char* msg) {
    g_thrown_class = static_cast<FakeClass*>(cls)->name;
    g_thrown_msg = msg;
    return 0;
}
void* JNIEnv::GetPrimitiveArrayCritical(jarray a, jboolean*) { return static_cast<FakeArray*>(a)->bytes.data(); }
void JNIEnv::ReleasePrimitiveArrayCritical(jarray, void*, jint) {}
jint* JNIEnv::GetIntArrayElements(jintArray a, jboolean*) { return (jint*)static_cast<FakeArray*>(a)->bytes.data(); }
void JNIEnv::ReleaseIntArrayElements(jintArray, jint*, jint) {}
jfloat* JNIEnv::GetFloatArrayElements(jfloatArray a, jboolean*) {
    return (jfloat*)static_cast<FakeArray*>(a)->bytes.data();
}
void JNIEnv::ReleaseFloatArrayElements(jfloatArray, jfloat*, jint) {}
jlong* JNIEnv::GetLongArrayElements(jlongArray a, jboolean*) { return (jlong*)static_cast<FakeArray*>(a)->bytes.data(); }
void JNIEnv::ReleaseLongArrayElements(jlongArray, jlong*, jint) {}
jobject JNIEnv::GetObjectArrayElement(jobjectArray a, jsize i) {
    return reinterpret_cast<jobject*>(static_cast<FakeArray*>(a)->bytes.data())[i];
}
jsize JNIEnv::GetArrayLength(jarray a) { return static_cast<FakeArray*>(a)->len; }
void JNIEnv::GetFloatArrayRegion(jfloatArray a, jsize s, jsize n, jfloat* b) {
    memcpy(b, static_cast<FakeArray*>(a)->bytes.data() + 4 * s, 4 * (size_t)n);
}
void JNIEnv::GetIntArrayRegion(jintArray a, jsize s, jsize n, jint* b) {
    memcpy(b, static_cast<FakeArray*>(a)->bytes.data() + 4 * s, 4 * (size_t)n);
}
jintArray JNIEnv::NewIntArray(jsize n) {
    FakeArray* a = new FakeArray();
    a->bytes.resize(4 * (size_t)n);
    a->len = n;
    return a;
}
void JNIEnv::SetIntArrayRegion(jintArray a, jsize s, jsize n, const jint* b) {
    memcpy(static_cast<FakeArray*>(a)->bytes.data() + 4 * s, b, 4 * (size_t)n);
}
const char* JNIEnv::GetStringUTFChars(jstring s, jboolean*) { return static_cast<FakeString*>(s)->s.c_str(); }
void JNIEnv::ReleaseStringUTFChars(jstring, const char*) {}

extern "C" {
void Java_com_epicmonstrosity_brewference_gpu_Brew_init(JNIEnv*, jclass, jint);
void Java_com_epicmonstrosity_brewference_gpu_Brew_matmul(JNIEnv*, jclass, jfloatArray, jfloatArray, jlong, jlong, jint,
                                                          jint);
jlong Java_com_epicmonstrosity_brewference_gpu_Brew_loadGguf(JNIEnv*, jclass, jstring, jint);
}

static FakeArray* floats(jsize n) {
    FakeArray* a = new FakeArray();
    a->bytes.assign(4 * (size_t)n, 0);
    a->len = n;
    return a;
}

static void report(const char* what) {
    printf("%s: %s | %s\n", what, g_thrown_class.c_str(), g_thrown_msg.c_str());
    g_thrown_class.clear();
    g_thrown_msg.clear();
}

int main(int argc, char** argv) {
    JNIEnv env;
    // Linear.matmul with null weights: IllegalArgumentException before any device work
    Java_com_epicmonstrosity_brewference_gpu_Brew_matmul(&env, nullptr, floats(4), floats(32), 0, 0, 32, 4);
    report("matmul_null_weights");
    // null arrays: the glue's own check
    Java_com_epicmonstrosity_brewference_gpu_Brew_matmul(&env, nullptr, nullptr, floats(32), 0, 0, 32, 4);
    report("matmul_null_arrays");
    // a file that is not a GGUF checkpoint: IOException
    FakeString path;
    path.s = argc > 1 ? argv[1] : "/nonexistent.gguf";
    jlong m = Java_com_epicmonstrosity_brewference_gpu_Brew_loadGguf(&env, nullptr, &path, 1);
    report(m ? "load_gguf_unexpected_model" : "load_gguf_bad_file");
    // device selection without a GPU: IllegalStateException (no CPU path)
    Java_com_epicmonstrosity_brewference_gpu_Brew_init(&env, nullptr, 0);
    report("init");
    return 0;
}
