// brew_jni.cpp — JNI glue between the Java reference's classes and the C ABI
// (include/brew.h).  Java side: class
// com.epicmonstrosity.brewference.gpu.Brew, a class of static native methods
// that the reference's Linear, loader and ModelRunner call.  Built into
// libbrew.so by brewference_b200/build.py when a JDK's jni.h is found
// (JAVA_HOME).
//
// Errors become the Java exceptions the reference throws for the same
// conditions: BREW_ERR_INVALID_ARG -> IllegalArgumentException
// (transformer/math/Linear.java:67-74), BREW_ERR_IO -> java.io.IOException
// (gguf/GgufWeightsLoader.java:76-78), everything else ->
// IllegalStateException (Linear.java:46-50, runtime/ModelRunner.java:208-216).
#include <jni.h>

#include <cstdint>
#include <vector>

#include "brew.h"

namespace {

void throw_for(JNIEnv* env, int rc) {
    char msg[1024];
    brew_last_error(msg, sizeof(msg));
    const char* cls = rc == BREW_ERR_INVALID_ARG ? "java/lang/IllegalArgumentException"
                      : rc == BREW_ERR_IO        ? "java/io/IOException"
                                                 : "java/lang/IllegalStateException";
    jclass c = env->FindClass(cls);
    if (c) env->ThrowNew(c, msg);
}

// Pins a primitive array for the duration of one C call.
template <typename J, typename T>
struct Pinned {
    JNIEnv* env;
    J arr;
    T* p;
    Pinned(JNIEnv* e, J a) : env(e), arr(a), p(a ? static_cast<T*>(e->GetPrimitiveArrayCritical(a, nullptr)) : nullptr) {}
    ~Pinned() {
        if (p) env->ReleasePrimitiveArrayCritical(arr, p, 0);
    }
};

}  // namespace

extern "C" {

JNIEXPORT void JNICALL Java_com_epicmonstrosity_brewference_gpu_Brew_init(JNIEnv* env, jclass, jint device) {
    const int rc = brew_init(device);
    if (rc) throw_for(env, rc);
}

// Packed GGUF bytes of a tensor (all layers concatenated) -> device handle.
JNIEXPORT jlong JNICALL Java_com_epicmonstrosity_brewference_gpu_Brew_uploadTensor(JNIEnv* env, jclass, jint type,
                                                                                   jbyteArray bytes, jlong n) {
    brew_tensor t = nullptr;
    int rc;
    {
        Pinned<jbyteArray, jbyte> b(env, bytes);
        rc = brew_tensor_upload(type, b.p, n, &t);
    }
    if (rc) throw_for(env, rc);
    return reinterpret_cast<jlong>(t);
}

JNIEXPORT void JNICALL Java_com_epicmonstrosity_brewference_gpu_Brew_freeTensor(JNIEnv*, jclass, jlong h) {
    brew_tensor_free(reinterpret_cast<brew_tensor>(h));
}

// Linear.matmul(output, input, weights, weightsOffset, inputSize, outputSize)
JNIEXPORT void JNICALL Java_com_epicmonstrosity_brewference_gpu_Brew_matmul(JNIEnv* env, jclass, jfloatArray out,
                                                                            jfloatArray in, jlong w, jlong off,
                                                                            jint inputSize, jint outputSize) {
    if (!out || !in) {
        jclass c = env->FindClass("java/lang/IllegalArgumentException");
        if (c) env->ThrowNew(c, "Input and output arrays cannot be null");
        return;
    }
    int rc;
    {
        Pinned<jfloatArray, float> o(env, out), i(env, in);
        rc = brew_matmul(o.p, i.p, reinterpret_cast<brew_tensor>(w), off, inputSize, outputSize);
    }
    if (rc) throw_for(env, rc);
}

// Model from uploaded tensors.  ints: arch, dim, hidden_dim, n_layers,
// n_heads, n_kv_heads, head_size, vocab_size, seq_len, sliding_window,
// bos, eos, tied, type_embed, type_output, type_q, type_k, type_v, type_o,
// type_gate, type_up, type_down; floats: eps, rope_base, rope_scale;
// tensors: embd, output, q, k, v, o, gate, up, down; vectors (null when
// absent): rms_att, rms_ffn, rms_final, post_att, post_ffn, rms_q, rms_k,
// q_bias, k_bias, v_bias.
JNIEXPORT jlong JNICALL Java_com_epicmonstrosity_brewference_gpu_Brew_modelCreate(JNIEnv* env, jclass, jintArray ints,
                                                                                  jfloatArray floats,
                                                                                  jlongArray tensors,
                                                                                  jobjectArray vectors, jint maxBatch) {
    brew_config c = {};
    {
        jint* v = env->GetIntArrayElements(ints, nullptr);
        c.arch = v[0]; c.dim = v[1]; c.hidden_dim = v[2]; c.n_layers = v[3]; c.n_heads = v[4];
        c.n_kv_heads = v[5]; c.head_size = v[6]; c.vocab_size = v[7]; c.seq_len = v[8]; c.sliding_window = v[9];
        c.bos_token = v[10]; c.eos_token = v[11]; c.tied_embeddings = v[12]; c.type_embed = v[13];
        c.type_output = v[14]; c.type_q = v[15]; c.type_k = v[16]; c.type_v = v[17]; c.type_o = v[18];
        c.type_gate = v[19]; c.type_up = v[20]; c.type_down = v[21];
        env->ReleaseIntArrayElements(ints, v, JNI_ABORT);
        jfloat* f = env->GetFloatArrayElements(floats, nullptr);
        c.eps = f[0]; c.rope_base = f[1]; c.rope_scale = f[2];
        env->ReleaseFloatArrayElements(floats, f, JNI_ABORT);
    }
    brew_model_weights w = {};
    {
        jlong* t = env->GetLongArrayElements(tensors, nullptr);
        brew_tensor* dst[] = {&w.token_embd, &w.output, &w.wq, &w.wk, &w.wv, &w.wo, &w.w_gate, &w.w_up, &w.w_down};
        for (int i = 0; i < 9; ++i) *dst[i] = reinterpret_cast<brew_tensor>(t[i]);
        env->ReleaseLongArrayElements(tensors, t, JNI_ABORT);
    }
    const float** vdst[] = {&w.rms_att, &w.rms_ffn, &w.rms_final, &w.post_att, &w.post_ffn,
                            &w.rms_q,   &w.rms_k,   &w.q_bias,    &w.k_bias,   &w.v_bias};
    std::vector<std::vector<float>> keep(10);
    for (int i = 0; i < 10; ++i) {
        jfloatArray a = static_cast<jfloatArray>(env->GetObjectArrayElement(vectors, i));
        if (!a) continue;
        keep[i].resize(env->GetArrayLength(a));
        env->GetFloatArrayRegion(a, 0, (jsize)keep[i].size(), keep[i].data());
        *vdst[i] = keep[i].data();
    }
    brew_model m = nullptr;
    const int rc = brew_model_create(&c, &w, maxBatch, &m);   // copies the vectors to the device
    if (rc) {
        throw_for(env, rc);
        return 0;
    }
    return reinterpret_cast<jlong>(m);
}

// GgufCheckpointLoader.loadWeights + GgufWeightsLoader.load in one call: the
// checkpoint's packed blocks go from the file to HBM (brew_model_load_gguf).
JNIEXPORT jlong JNICALL Java_com_epicmonstrosity_brewference_gpu_Brew_loadGguf(JNIEnv* env, jclass, jstring path,
                                                                               jint maxBatch) {
    if (!path) {
        jclass c = env->FindClass("java/lang/IllegalArgumentException");
        if (c) env->ThrowNew(c, "path cannot be null");
        return 0;
    }
    const char* p = env->GetStringUTFChars(path, nullptr);
    brew_model m = nullptr;
    const int rc = brew_model_load_gguf(p, maxBatch, &m);
    env->ReleaseStringUTFChars(path, p);
    if (rc) {
        throw_for(env, rc);
        return 0;
    }
    return reinterpret_cast<jlong>(m);
}

JNIEXPORT void JNICALL Java_com_epicmonstrosity_brewference_gpu_Brew_modelFree(JNIEnv*, jclass, jlong m) {
    brew_model_free(reinterpret_cast<brew_model>(m));
}

// brew_model_set_prefill: 0 token by token (default), 1 batched (tcgen05 GEMM).
JNIEXPORT void JNICALL Java_com_epicmonstrosity_brewference_gpu_Brew_setPrefill(JNIEnv* env, jclass, jlong m,
                                                                                jint mode) {
    const int rc = brew_model_set_prefill(reinterpret_cast<brew_model>(m), mode);
    if (rc) throw_for(env, rc);
}

// TransformerGraph.forward(token, pos) + Kernels.argMax; logits copied into
// `logits` when it is not null.  Returns the argmax id.
JNIEXPORT jint JNICALL Java_com_epicmonstrosity_brewference_gpu_Brew_forward(JNIEnv* env, jclass, jlong m, jint token,
                                                                             jint pos, jfloatArray logits) {
    int32_t tok = token, p = pos, am = -1;
    int rc;
    {
        Pinned<jfloatArray, float> lg(env, logits);
        rc = brew_model_forward(reinterpret_cast<brew_model>(m), &tok, &p, 1, lg.p, &am);
    }
    if (rc) throw_for(env, rc);
    return am;
}

// Greedy generation with ModelRunner's token order; returns the new ids
// (maxNew <= 0: up to the rest of the context).
JNIEXPORT jintArray JNICALL Java_com_epicmonstrosity_brewference_gpu_Brew_generate(JNIEnv* env, jclass, jlong m,
                                                                                   jintArray prompt, jint maxNew) {
    const jsize n = env->GetArrayLength(prompt);
    brew_config c = {};
    const int rc0 = brew_model_config(reinterpret_cast<brew_model>(m), &c);
    if (rc0) {
        throw_for(env, rc0);
        return nullptr;
    }
    const int cap = maxNew > 0 ? maxNew : (c.seq_len > n ? c.seq_len - n : 0);
    std::vector<int32_t> pr(n), out(cap > 0 ? cap : 1);
    env->GetIntArrayRegion(prompt, 0, n, reinterpret_cast<jint*>(pr.data()));
    int32_t n_out = 0;
    const int rc = brew_session_generate(reinterpret_cast<brew_model>(m), pr.data(), n, maxNew, out.data(), &n_out);
    if (rc) {
        throw_for(env, rc);
        return nullptr;
    }
    jintArray res = env->NewIntArray(n_out);
    env->SetIntArrayRegion(res, 0, n_out, reinterpret_cast<jint*>(out.data()));
    return res;
}

}  // extern "C"
