/* Test-only stand-in for the JDK's <jni.h>: the JNI types and the JNIEnv
 * member functions that brewference_b200/csrc/jni/brew_jni.cpp uses, with the
 * signatures of the JNI specification.  No JDK exists in this image; the
 * member functions are defined by tests/jni_stub/fake_env.cpp, which records
 * thrown exceptions and serves arrays from host memory, so the glue can be
 * compiled, linked against libbrew.so and exercised on the CPU. */
#ifndef BREW_TEST_JNI_H
#define BREW_TEST_JNI_H

#include <stdint.h>

typedef int32_t jint;
typedef int64_t jlong;
typedef int8_t jbyte;
typedef float jfloat;
typedef uint8_t jboolean;
typedef jint jsize;

struct _jobject {};
typedef _jobject* jobject;
typedef jobject jclass;
typedef jobject jstring;
typedef jobject jarray;
typedef jarray jbyteArray;
typedef jarray jfloatArray;
typedef jarray jintArray;
typedef jarray jlongArray;
typedef jarray jobjectArray;
typedef jobject jthrowable;

#define JNIEXPORT __attribute__((visibility("default")))
#define JNICALL
#define JNI_ABORT 2

struct JNIEnv {
    jclass FindClass(const char* name);
    jint ThrowNew(jclass cls, const char* msg);
    void* GetPrimitiveArrayCritical(jarray a, jboolean* is_copy);
    void ReleasePrimitiveArrayCritical(jarray a, void* p, jint mode);
    jint* GetIntArrayElements(jintArray a, jboolean* is_copy);
    void ReleaseIntArrayElements(jintArray a, jint* p, jint mode);
    jfloat* GetFloatArrayElements(jfloatArray a, jboolean* is_copy);
    void ReleaseFloatArrayElements(jfloatArray a, jfloat* p, jint mode);
    jlong* GetLongArrayElements(jlongArray a, jboolean* is_copy);
    void ReleaseLongArrayElements(jlongArray a, jlong* p, jint mode);
    jobject GetObjectArrayElement(jobjectArray a, jsize i);
    jsize GetArrayLength(jarray a);
    void GetFloatArrayRegion(jfloatArray a, jsize start, jsize len, jfloat* buf);
    void GetIntArrayRegion(jintArray a, jsize start, jsize len, jint* buf);
    jintArray NewIntArray(jsize len);
    void SetIntArrayRegion(jintArray a, jsize start, jsize len, const jint* buf);
    const char* GetStringUTFChars(jstring s, jboolean* is_copy);
    void ReleaseStringUTFChars(jstring s, const char* p);
};

#endif
